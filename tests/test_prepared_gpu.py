"""Prepared GEMM calls (b2g_prepare_gemm / b2g_prepared_run through
ops.PreparedGemm) on a B200: bit-identical to the direct entry points for every
kind and both kernels (persistent and small-M), reading the operands' current
contents on every run, on any stream, with less host work per call."""

from __future__ import annotations

import time

import pytest
import torch

from gfx950_gluon_tutorials_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def _f16(M, N, K, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = (torch.randn((M, K), generator=g, device="cuda") / K ** 0.5).to(dtype)
    b = (torch.randn((N, K), generator=g, device="cuda") / K ** 0.5).to(dtype)
    return a, b


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["fp16", "bf16"])
@pytest.mark.parametrize("shape", [(4096, 4096, 8192), (1000, 1200, 4096), (16, 4096, 1024)],
                         ids=lambda s: "x".join(map(str, s)))
def test_prepared_f16_matches_direct(cuda_device, dtype, shape):
    M, N, K = shape
    a, b = _f16(M, N, K, dtype, M + N + K)
    ref = ops.gemm_f16(a, b)
    c = torch.empty_like(ref)
    p = ops.prepare_gemm_f16(a, b, c)
    assert p() is c
    torch.cuda.synchronize()
    assert torch.equal(c, ref)
    # new contents in the same storage are read by the next run
    a.mul_(-1.0)
    b[0].zero_()
    p()
    ops.check_status()
    assert torch.equal(c, ops.gemm_f16(a, b))
    p.close()


def test_prepared_e5m2_both_forms(cuda_device):
    M, N, K = 1024, 768, 2048
    g = torch.Generator(device="cuda").manual_seed(5)
    a = (torch.rand((M, K), generator=g, device="cuda").half() - 0.5).to(torch.float8_e5m2)
    b = (torch.rand((N, K), generator=g, device="cuda").half() - 0.5).to(torch.float8_e5m2)
    ea = torch.randint(125, 130, (M, K // 32), generator=g, device="cuda").to(torch.uint8)
    eb = torch.randint(125, 130, (N, K // 32), generator=g, device="cuda").to(torch.uint8)
    c = torch.empty((M, N), dtype=torch.float16, device="cuda")
    assert torch.equal(ops.prepare_gemm_f8(a, b, c)(), ops.gemm_f8(a, b))
    cs = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    ref = ops.gemm_f8(a, b, a_scales=ea, b_scales=eb, out_dtype=torch.bfloat16)
    assert torch.equal(ops.prepare_gemm_f8(a, b, cs, a_scales=ea, b_scales=eb)(), ref)
    blocked = ops.prepare_gemm_f8(a, b, torch.empty_like(cs), a_scales=ops.block_scales(ea),
                                  b_scales=ops.block_scales(eb))
    assert torch.equal(blocked(), ref)
    ops.check_status()


@pytest.mark.parametrize("shape", [(4096, 4096, 8192), (300, 704, 1024)],
                         ids=lambda s: "x".join(map(str, s)))
def test_prepared_mxf4_matches_direct_on_another_stream(cuda_device, shape):
    M, N, K = shape
    g = torch.Generator(device="cuda").manual_seed(7)
    qa, sa = ops.quantize_mxfp4(torch.randn((M, K), generator=g, device="cuda"))
    qb, sb = ops.quantize_mxfp4(torch.randn((N, K), generator=g, device="cuda"))
    ref = ops.gemm_mxf4(qa, qb, sa, sb)
    c = torch.empty_like(ref)
    p = ops.prepare_gemm_mxf4(qa, qb, sa, sb, c)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            p()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    ops.check_status()
    assert torch.equal(c, ref)


def test_prepared_rejects_operands_it_would_copy(cuda_device):
    a = torch.randn((64, 200), device="cuda").half()[:, :100]   # 200-byte rows: not 16-aligned
    b = torch.randn((64, 100), device="cuda").half()
    with pytest.raises(ValueError):
        ops.prepare_gemm_f16(a, b)
    c_col_major = torch.empty((64, 64), device="cuda").half().T   # unit row stride
    with pytest.raises(ValueError):
        ops.prepare_gemm_f16(b, b, c_col_major)


def test_prepared_runs_need_the_device_they_were_planned_on(cuda_device):
    a, b = _f16(128, 256, 64, torch.float16, 1)
    p = ops.prepare_gemm_f16(a, b)
    if torch.cuda.device_count() > 1:
        with torch.cuda.device(1):
            rc = _lib.lib().b2g_prepared_run(p._h, None)
        assert rc == _lib.ENODEVICE
    p()
    torch.cuda.synchronize()
    ops.check_status()


def test_prepared_calls_take_less_host_time(cuda_device):
    """Small-M problem (host-bound): 300 back-to-back launches through the
    prepared handle against 300 direct calls through ops."""
    a, b = _f16(16, 1024, 512, torch.float16, 3)
    c = torch.empty((16, 1024), dtype=torch.float16, device="cuda")
    p = ops.prepare_gemm_f16(a, b, c)
    for _ in range(20):
        p()
        ops.gemm_f16(a, b, c)
    torch.cuda.synchronize()

    def host_us(fn):
        t0 = time.perf_counter()
        for _ in range(300):
            fn()
        t1 = time.perf_counter()
        torch.cuda.synchronize()
        return (t1 - t0) / 300 * 1e6

    direct = min(host_us(lambda: ops.gemm_f16(a, b, c)) for _ in range(3))
    prepared = min(host_us(p) for _ in range(3))
    ops.check_status()
    assert prepared < direct, (prepared, direct)


def test_calls_replay_from_a_cuda_graph(cuda_device):
    """Direct and prepared calls captured in a CUDA graph (the launches carry
    programmatic stream serialization) replay to the same bits as eager calls,
    and a replay reads the inputs' current contents."""
    a, b = _f16(1024, 2048, 4096, torch.float16, 11)
    g = torch.Generator(device="cuda").manual_seed(12)
    qa, sa = ops.quantize_mxfp4(torch.randn((512, 2048), generator=g, device="cuda"))
    qb, sb = ops.quantize_mxfp4(torch.randn((768, 2048), generator=g, device="cuda"))
    c1 = torch.empty((1024, 2048), dtype=torch.float16, device="cuda")
    c2 = torch.empty((512, 768), dtype=torch.bfloat16, device="cuda")
    p = ops.prepare_gemm_mxf4(qa, qb, sa, sb, c2)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):           # warm up on the capture stream (its workspace)
        ops.gemm_f16(a, b, c1)
        p()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        ops.gemm_f16(a, b, c1)
        p()
    a.mul_(0.5)
    graph.replay()
    torch.cuda.synchronize()
    ops.check_status()
    assert torch.equal(c1, ops.gemm_f16(a, b))
    assert torch.equal(c2, ops.gemm_mxf4(qa, qb, sa, sb))
