"""Attention forward on the B200: the sm_100a kernel through the C ABI against
the reference's golden outputs and the float64 oracle, with the reference's
own tolerance rule (kernels/attention/common.py:142, restated as
oracle.attention.check_output: atol = max(1e-3, 2 ULP x max|ref|), rtol 1e-3)."""

from __future__ import annotations

import glob
import os

import numpy as np
import pytest
import torch

from gfx950_gluon_tutorials_b200 import _lib, attention, ops
from oracle import attention as oa

pytestmark = pytest.mark.gpu

GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "attention_*.npz")))
TDT = {"float16": torch.float16, "bfloat16": torch.bfloat16}


def _to_bhsd(t, layout):
    return t if layout == "bhsd" else t.transpose(1, 2)


def _run(q, k, v, layout="bhsd", sm_scale=None, with_lse=False):
    order = (0, 1, 2) if layout == "bhsd" else (0, 2, 1)
    B, HQ, Sq = (q.shape[i] for i in order)
    lse = torch.full((B, HQ, Sq), float("nan"), device="cuda") if with_lse else None
    o = torch.full_like(q, float("nan"))
    attention.attention_fwd(q, k, v, o, sm_scale=sm_scale, layout=layout, lse=lse)
    ops.check_status()
    return o, lse


def _inputs(B, HQ, HK, Sq, Sk, D, dtype, layout, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)

    def rand(h, s):
        shape = (B, h, s, D) if layout == "bhsd" else (B, s, h, D)
        return torch.randn(shape, generator=g, device="cuda", dtype=torch.float32).to(dtype)

    return rand(HQ, Sq), rand(HK, Sk), rand(HK, Sk)


def _oracle(q, k, v, layout, sm_scale):
    f = [_to_bhsd(t, layout).float().cpu().numpy() for t in (q, k, v)]
    return oa.sdpa_ref(*f, sm_scale)


@pytest.mark.parametrize("path", GOLDEN, ids=lambda p: os.path.basename(p)[:-4])
def test_matches_reference_golden(cuda_device, path):
    z = np.load(path)
    dt = TDT[str(z["dtype"])]
    q, k, v = (torch.from_numpy(z[n].view(np.int16)).view(dt).cuda() for n in "qkv")
    o, _ = _run(q, k, v, sm_scale=float(z["sm_scale"]))
    ok, mx, mean = oa.check_output(o.float().cpu().numpy(), z["o_ref"], str(z["dtype"]))
    assert ok, f"max |diff| {mx:.3e}, mean {mean:.3e}"


SHAPES = [
    # B, HQ, HK, Sq, Sk, D
    (1, 2, 2, 128, 128, 128),
    (2, 4, 1, 256, 384, 128),     # GQA 4:1
    (1, 3, 3, 1, 1, 128),         # one query, one key
    (1, 2, 1, 77, 1000, 128),     # ragged both ways
    (3, 2, 2, 300, 129, 64),
    (1, 8, 2, 1024, 1024, 64),
    (1, 1, 1, 640, 4095, 128),
]


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
@pytest.mark.parametrize("layout", ["bhsd", "bshd"])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_matches_oracle(cuda_device, shape, layout, dtype):
    B, HQ, HK, Sq, Sk, D = shape
    q, k, v = _inputs(*shape, TDT[dtype], layout, seed=sum(shape))
    sm_scale = D ** -0.5
    o, lse = _run(q, k, v, layout, sm_scale, with_lse=True)
    o_ref, lse_ref = _oracle(q, k, v, layout, sm_scale)
    ok, mx, mean = oa.check_output(_to_bhsd(o, layout).float().cpu().numpy(), o_ref, dtype)
    assert ok, f"max |diff| {mx:.3e}, mean {mean:.3e}"
    np.testing.assert_allclose(lse.cpu().numpy(), lse_ref, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
def test_many_items_with_mixed_tile_counts(cuda_device, dtype):
    """More work items than SMs, where every other item holds one query tile
    (Sq = 300 = 256 + 44): the persistent CTAs' per-tile barrier phases must
    stay in step across items of both kinds."""
    shape = (2, 100, 20, 300, 200, 64)
    B, HQ, HK, Sq, Sk, D = shape
    q, k, v = _inputs(*shape, TDT[dtype], "bshd", seed=123)
    o, lse = _run(q, k, v, "bshd", D ** -0.5, with_lse=True)
    o_ref, lse_ref = _oracle(q, k, v, "bshd", D ** -0.5)
    ok, mx, mean = oa.check_output(_to_bhsd(o, "bshd").float().cpu().numpy(), o_ref, dtype)
    assert ok, f"max |diff| {mx:.3e}, mean {mean:.3e}"
    np.testing.assert_allclose(lse.cpu().numpy(), lse_ref, rtol=1e-4, atol=1e-4)


def test_large_scores_and_moving_max(cuda_device):
    """Scores spread over hundreds of units in log2: the running max moves
    often and by large steps, exercising the O rescale; rows where a late key
    dominates included."""
    B, HQ, HK, S, D = 1, 2, 2, 1024, 128
    q, k, v = _inputs(B, HQ, HK, S, S, D, torch.bfloat16, "bhsd", seed=11)
    ramp = torch.linspace(0.2, 3.0, S, device="cuda").view(1, 1, S, 1)
    k = (k.float() * ramp).to(torch.bfloat16)
    q = (q.float() * 2).to(torch.bfloat16)
    o, lse = _run(q, k, v, "bhsd", 1.0, with_lse=True)
    o_ref, lse_ref = _oracle(q, k, v, "bhsd", 1.0)
    ok, mx, _ = oa.check_output(o.float().cpu().numpy(), o_ref, "bfloat16")
    assert ok, f"max |diff| {mx:.3e}"
    np.testing.assert_allclose(lse.cpu().numpy(), lse_ref, rtol=1e-4, atol=1e-3)


def test_run_gluon_attention_dropin(cuda_device):
    """The reference launcher's call shape: input_helper problem, o preallocated."""
    for layout in ("bhsd", "bshd"):
        q, k, v, md = attention.input_helper(1, 4, 2, 512, 512, 128, torch.bfloat16, layout)
        o = torch.empty_like(q)
        attention.run_gluon_attention(q, k, v, o, md)
        ops.check_status()
        o_ref, _ = _oracle(q, k, v, layout, md.sm_scale)
        ok, mx, _ = oa.check_output(_to_bhsd(o, layout).float().cpu().numpy(), o_ref, "bfloat16")
        assert ok, f"{layout}: max |diff| {mx:.3e}"


def test_noncontiguous_output_and_strided_inputs(cuda_device):
    """q sliced out of a packed qkv buffer (bshd), o a strided view."""
    B, S, H, D = 2, 200, 4, 64
    g = torch.Generator(device="cuda").manual_seed(9)
    qkv = torch.randn((B, S, 3, H, D), generator=g, device="cuda").to(torch.float16)
    q, k, v = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
    o_big = torch.zeros((B, S, H, 2 * D), dtype=torch.float16, device="cuda")
    o = o_big[..., :D]
    attention.attention_fwd(q, k, v, o, layout="bshd")
    ops.check_status()
    o_ref, _ = _oracle(q, k, v, "bshd", D ** -0.5)
    ok, mx, _ = oa.check_output(o.transpose(1, 2).float().cpu().numpy(), o_ref, "float16")
    assert ok, f"max |diff| {mx:.3e}"
    assert bool((o_big[..., D:] == 0).all()), "wrote outside the output view"


def test_deterministic(cuda_device):
    q, k, v = _inputs(1, 4, 4, 512, 700, 128, torch.bfloat16, "bhsd", seed=5)
    a, _ = _run(q, k, v)
    b, _ = _run(q, k, v)
    assert torch.equal(a, b)


def test_bench_config_sampled_rows(cuda_device):
    """The reference bench's default problem (B=1, HQ=HK=64, S=8192, D=128,
    bf16, bhsd): rows sampled from four heads checked against the oracle."""
    B, H, S, D = 1, 64, 8192, 128
    q, k, v, md = attention.input_helper(B, H, H, S, S, D, torch.bfloat16, "bhsd")
    o = torch.empty_like(q)
    attention.run_gluon_attention(q, k, v, o, md)
    ops.check_status()
    rows = torch.tensor([0, 1, 127, 128, 4095, 5000, 8064, 8191])
    for h in (0, 17, 42, 63):
        qs = q[:, h:h + 1, rows].float().cpu().numpy()
        ks = k[:, h:h + 1].float().cpu().numpy()
        vs = v[:, h:h + 1].float().cpu().numpy()
        o_ref, _ = oa.sdpa_ref(qs, ks, vs, md.sm_scale)
        got = o[:, h:h + 1, rows].float().cpu().numpy()
        ok, mx, _ = oa.check_output(got, o_ref, "bfloat16")
        assert ok, f"head {h}: max |diff| {mx:.3e}"


def test_status_stays_clear_and_errors_raise(cuda_device):
    q = torch.zeros((1, 2, 128, 96), dtype=torch.float16, device="cuda")
    with pytest.raises(_lib.B2GError):
        attention.attention_fwd(q, q, q)  # head dim 96
    assert int(ops.status_tensor(q.device).item()) == 0


def test_poly_exp2_relative_error_bound(cuda_device):
    """The FMHA's FMA-pipe exponential (poly_exp2 and its packed two-lane form)
    against float64 2^x and CUDA's exp2f: relative error <= 7.5e-5 on
    [-125.5, 8]; inputs at or below the -126 clamp (masked keys are -inf) give
    a tiny non-negative finite value; both forms agree bit for bit."""
    dense = torch.linspace(-125.5, 8.0, 4_000_001, dtype=torch.float64).float()
    steps = torch.arange(-125.5, 8.25, 0.25, dtype=torch.float64).float()   # f = 0, +-0.25, 0.5
    nudged = torch.cat([steps.nextafter(torch.tensor(-1e9)), steps.nextafter(torch.tensor(1e9))])
    x_in = torch.cat([dense, steps, nudged.clamp(-125.5, 8.0)]).cuda()
    x_low = torch.tensor([-126.0, -126.5, -150.0, -1e30, float("-inf")], device="cuda")
    x = torch.cat([x_in, x_low])
    ys, yp, ye = (torch.empty_like(x) for _ in range(3))
    rc = _lib.lib().b2g_selftest_poly_exp2(x.data_ptr(), ys.data_ptr(), yp.data_ptr(),
                                           ye.data_ptr(), x.numel(),
                                           torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.OK
    torch.cuda.synchronize()
    assert torch.equal(ys.view(torch.int32), yp.view(torch.int32)), "pair form differs"
    n = x_in.numel()
    exact = torch.exp2(x_in.double())
    rel = ((ys[:n].double() - exact).abs() / exact).max().item()
    rel_f = ((ys[:n].double() - ye[:n].double()).abs() / ye[:n].double()).max().item()
    assert rel <= 7.5e-5, f"max relative error vs 2^x {rel:.3e}"
    assert rel_f <= 7.6e-5, f"max relative error vs exp2f {rel_f:.3e}"
    low = ys[n:]
    assert bool(torch.isfinite(low).all()) and bool((low >= 0).all())
    assert bool((low < 2.0 ** -125).all())
