"""Host-side logic of the multi-GPU path on CPU ranks (gloo, world size 2 and 4):
N-sharding covers every column exactly once, gathered slabs assemble to the
full product, and a rank that fails is reported instead of hanging."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gfx950_gluon_tutorials_b200.shard import assemble, chunk_rows, gather_slabs, shard_range


@pytest.mark.parametrize("n,world", [(4096, 1), (53248, 2), (53248, 8), (700, 3), (300, 4)])
def test_shard_ranges_partition_columns(n, world):
    seen = []
    for r in range(world):
        a, b = shard_range(n, world, r)
        assert a <= b and (a % 256 == 0)
        seen.extend(range(a, b))
    assert seen == list(range(n))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, queue, fail_rank):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=20))
    try:
        g = torch.Generator().manual_seed(0)
        M, N, K = 64, 256 * world, 96
        a = torch.randn(M, K, generator=g)
        b = torch.randn(N, K, generator=g)
        lo, hi = shard_range(N, world, rank)
        if rank == fail_rank:
            raise RuntimeError("injected rank failure")
        c_local = a @ b[lo:hi].T                        # this rank's slab
        slabs = gather_slabs(c_local)
        full = assemble(slabs)
        ok = torch.allclose(full, a @ b.T, atol=1e-4, rtol=1e-4)
        queue.put((rank, "ok" if ok else "mismatch"))
    except Exception as e:  # noqa: BLE001
        queue.put((rank, f"error: {e}"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _run(world, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, fail_rank))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    out = {}
    while not q.empty():
        r, msg = q.get()
        out[r] = msg
    return out


@pytest.mark.parametrize("world", [2, 4])
def test_gathered_slabs_assemble_the_full_product(world):
    out = _run(world)
    assert out == {r: "ok" for r in range(world)}


def test_a_failing_rank_is_reported_not_hung():
    out = _run(2, fail_rank=1)
    assert out.get(1, "").startswith("error: injected")
    # the surviving rank's collective ends with an error within the group timeout
    assert out.get(0, "").startswith("error")


@pytest.mark.parametrize("m,chunks", [(4096, 4), (1000, 3), (256, 8), (16384, 5)])
def test_chunk_rows_cover_whole_tiles(m, chunks):
    pieces = chunk_rows(m, chunks)
    assert pieces[0][0] == 0 and pieces[-1][1] == m
    for (lo, hi), (lo2, _) in zip(pieces, pieces[1:]):
        assert hi == lo2 and lo % 256 == 0
    assert len(pieces) <= chunks


def _gather_worker(rank, world, port, queue):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    from gfx950_gluon_tutorials_b200 import shard
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=20))
    try:
        g = torch.Generator().manual_seed(0)
        M, N, K = 64, 256 * world, 96
        a = torch.randn(M, K, generator=g)
        b = torch.randn(N, K, generator=g)
        lo, hi = shard.shard_range(N, world, rank)
        shard.P2P_MAX_WORLD = 1   # above it: the GEMM-then-gather path (no GPU needed)

        def matmul(x, y, out):
            out.copy_(x @ y.T)
            return out

        slabs = shard.gemm_gather(matmul, a, b[lo:hi], out_dtype=torch.float32)
        ok = tuple(slabs.shape) == (world, M, hi - lo) and torch.allclose(
            shard.assemble(slabs), a @ b.T, atol=1e-4, rtol=1e-4)
        queue.put((rank, "ok" if ok else "mismatch"))
    except Exception as e:  # noqa: BLE001
        queue.put((rank, f"error: {e}"))
    finally:
        dist.destroy_process_group()


def test_gemm_gather_large_world_path_gathers_every_slab():
    """Above P2P_MAX_WORLD ranks, `gemm_gather` runs the whole slab GEMM and
    then the all-gather; every rank ends with all slabs in rank order."""
    world = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    out = {}
    while not q.empty():
        r, msg = q.get()
        out[r] = msg
    assert out == {r: "ok" for r in range(world)}
