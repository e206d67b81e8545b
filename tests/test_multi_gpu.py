"""The overlapped GEMM + gather on two GPUs (skipped with fewer): every rank's
slab lands in every rank's symmetric buffer by peer-to-peer copies, and the
result equals the NCCL all-gather of the same chunked GEMM bit for bit."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime
    import torch.distributed as dist
    from gfx950_gluon_tutorials_b200 import ops
    from gfx950_gluon_tutorials_b200.shard import chunk_rows, gather_slabs, gemm_gather_p2p
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        M, N, K = 1000, 512, 1024
        a = torch.randn(M, K, generator=torch.Generator().manual_seed(0)).half().cuda()
        b = torch.randn(N, K, generator=torch.Generator().manual_seed(rank + 1)).half().cuda()
        local = torch.cat([ops.gemm_f16(a[lo:hi], b) for lo, hi in chunk_rows(M, 3)])
        ref = gather_slabs(local)
        results = []
        for _ in range(2):  # the reused buffer is rewritten correctly
            got = gemm_gather_p2p(lambda x, y, out: ops.gemm_f16(x, y, out), a, b, chunks=3)
            torch.cuda.synchronize()
            results.append(torch.equal(got, ref))
        ops.check_status()
        queue.put((rank, "ok" if all(results) else f"mismatch {results}"))
    except Exception as e:  # noqa: BLE001
        queue.put((rank, f"error: {e}"))
    finally:
        dist.destroy_process_group()


def test_p2p_gather_equals_nccl_gather():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert all(v == "ok" for v in results.values()), results
