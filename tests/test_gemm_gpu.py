"""GEMM parity on a B200: the sm_100a kernels (through the C ABI) against the
CPU oracle on the same seeded inputs, plus the golden vectors the reference's
own functions produced.

Tolerances: normalised max-abs error max|C - C_ref| / max|C_ref| <= 1e-2 for
FP16/BF16 and <= 3e-2 for BF8/MXFP4, plus the reference's own
allclose(atol=0.1, rtol=0) check (kernels/gemm/intra_wave/*/bench.py)."""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import golden

from gfx950_gluon_tutorials_b200 import _lib, a4w4, a8w8, a16w16, ops
from oracle import mx

pytestmark = pytest.mark.gpu

TOL_F16 = 1e-2
TOL_F8 = 3e-2


def bits16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def as_f32(t: torch.Tensor) -> np.ndarray:
    return t.float().cpu().numpy()


def assert_close(c: np.ndarray, ref: np.ndarray, tol: float, ref_atol: bool = True):
    """Normalised max-abs error within `tol`; with `ref_atol`, also the reference's
    allclose(atol=0.1, rtol=0). That absolute check only means something for the
    reference's own input recipes (rand - 0.5, random nibbles), whose outputs are
    small; N(0,1)-scaled operands give outputs near 100 where one bf16 ulp is 0.5."""
    err = mx.normalised_max_abs(c, ref)
    assert err <= tol, f"normalised max-abs error {err:.3e} > {tol}"
    if ref_atol:
        assert np.allclose(c, ref, atol=1e-1, rtol=0), "reference allclose(atol=0.1) failed"


@pytest.fixture(params=[
    dict(pair=1, sk=3, min_sk=4, units=0),
    dict(pair=0, sk=3, min_sk=4, units=0),
    dict(pair=1, sk=1, min_sk=4, units=0),
    dict(pair=0, sk=1, min_sk=4, units=0),
    dict(pair=1, sk=2, min_sk=1, units=0),
    dict(pair=0, sk=0, min_sk=4, units=0),
    dict(pair=1, sk=1, min_sk=1, units=5),   # few units: deep stream-K splits
    dict(pair=0, sk=2, min_sk=1, units=7),
    dict(pair=1, sk=3, min_sk=1, units=9),
    dict(pair=1, sk=4, min_sk=4, units=0),   # leftover tiles as half-width tiles
    dict(pair=0, sk=4, min_sk=4, units=0),
    dict(pair=1, sk=4, min_sk=1, units=13),  # few units: halves fit only sometimes
    dict(pair=1, sk=3, min_sk=4, units=3, serp=0),  # every tile walks K forwards
    dict(pair=0, sk=1, min_sk=4, units=5, serp=0),
], ids=lambda d: f"pair{d['pair']}-sk{d['sk']}-min{d['min_sk']}-u{d['units']}"
                 + ("-fwd" if d.get("serp", 1) == 0 else ""))
def sched(request, cuda_device):
    """Main-kernel schedule variants; the small-M swap-AB kernel is switched off
    so that these cases keep exercising the persistent kernel."""
    keys = {"pair": _lib.OPT_PAIR, "sk": _lib.OPT_SK_MODE, "min_sk": _lib.OPT_MIN_SK_ITERS,
            "units": _lib.OPT_MAX_UNITS, "skinny": _lib.OPT_SKINNY_MAX_M,
            "serp": _lib.OPT_SERPENTINE}
    old = {k: _lib.get_option(v) for k, v in keys.items()}
    for k, v in dict(dict(serp=1), **request.param, skinny=0).items():
        _lib.set_option(keys[k], v)
    yield request.param
    for k, v in old.items():
        _lib.set_option(keys[k], v)
    ops.check_status(cuda_device)


F16_SHAPES = [(128, 256, 64), (256, 512, 512), (300, 700, 200), (1000, 1000, 1024),
              (64, 2048, 4096), (2048, 96, 136)]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["fp16", "bf16"])
@pytest.mark.parametrize("shape", F16_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_a16w16_matches_oracle(sched, dtype, shape):
    M, N, K = shape
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N * 3 + K)
    a = torch.rand((M, K), generator=g, device="cuda", dtype=torch.float32).to(dtype) - 0.5
    b_t = torch.rand((N, K), generator=g, device="cuda", dtype=torch.float32).to(dtype) - 0.5
    c = ops.gemm_f16(a, b_t)
    ops.check_status()
    if dtype == torch.float16:
        ref = mx.gemm_f16_ref(a.cpu().numpy(), b_t.cpu().numpy(), "f16").astype(np.float32)
    else:
        ref = mx.bf16_bits_to_f32(mx.gemm_f16_ref(bits16(a), bits16(b_t), "bf16"))
    assert_close(as_f32(c), ref, TOL_F16)


@pytest.mark.parametrize("name,dtype", [("a16w16_f16_128x256x320.npz", torch.float16),
                                        ("a16w16_bf16_128x256x320.npz", torch.bfloat16)])
def test_a16w16_golden_via_reference_api(cuda_device, name, dtype):
    g = golden(name)
    if dtype == torch.float16:
        a = torch.from_numpy(g["a"]).cuda()
        b_t = torch.from_numpy(g["b_t"]).cuda()
        ref = g["c"].astype(np.float32)
    else:
        a = torch.from_numpy(g["a"].view(np.int16)).view(torch.bfloat16).cuda()
        b_t = torch.from_numpy(g["b_t"].view(np.int16)).view(torch.bfloat16).cuda()
        ref = mx.bf16_bits_to_f32(g["c"])
    c = a16w16.matmul(a, b_t.T)  # the reference bench passes b as a (K, N) view
    ops.check_status()
    assert c.dtype == dtype
    assert_close(as_f32(c), ref, TOL_F16)


def test_a16w16_explicit_c_and_strided_rows(cuda_device):
    M, N, K = 192, 320, 256
    a_store = torch.randn((M, K + 64), device="cuda", dtype=torch.float16)
    a = a_store[:, :K]                       # row stride K + 64
    b_t = torch.randn((N, K), device="cuda", dtype=torch.float16)
    c_store = torch.full((M, N + 8), float("nan"), device="cuda", dtype=torch.float16)
    c = c_store[:, :N]
    a16w16.matmul_kernel_only(a, b_t, c)
    ops.check_status()
    ref = mx.gemm_f16_ref(a.cpu().numpy(), b_t.cpu().numpy()).astype(np.float32)
    assert_close(as_f32(c), ref, TOL_F16, ref_atol=False)
    assert torch.isnan(c_store[:, N:]).all(), "wrote outside C"


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["fp16", "bf16"])
def test_a16w16_full_size_sampled_rows(cuda_device, dtype):
    """Config-1 size (4096 x 4096 x 8192), fp16 and bf16: the whole C against
    the oracle on a seeded sample of 256 rows, and against the exact GPU
    product for all rows."""
    M = N = 4096
    K = 8192
    g = torch.Generator(device="cuda").manual_seed(1)
    a = (torch.randn((M, K), generator=g, device="cuda") / K ** 0.5).to(dtype)
    b_t = (torch.randn((N, K), generator=g, device="cuda") / K ** 0.5).to(dtype)
    c = ops.gemm_f16(a, b_t)
    ops.check_status()
    assert c.dtype == dtype
    rows = torch.randperm(M, generator=torch.Generator().manual_seed(2))[:256].cuda()
    if dtype == torch.float16:
        ref = mx.gemm_f16_ref(a[rows].cpu().numpy(), b_t.cpu().numpy()).astype(np.float32)
    else:
        ref = mx.bf16_bits_to_f32(mx.gemm_f16_ref(bits16(a[rows]), bits16(b_t), "bf16"))
    assert_close(as_f32(c[rows]), ref, TOL_F16, ref_atol=False)
    full = (a.float() @ b_t.float().T)
    err = ((c.float() - full).abs().max() / full.abs().max()).item()
    assert err <= TOL_F16


def _gpu_normalised_err(c: torch.Tensor, ref: torch.Tensor) -> float:
    return ((c.float() - ref).abs().max() / ref.abs().max()).item()


def test_a8w8_scaled_cfg2_full_size(cuda_device):
    """BASELINE config 2 at its benched size, 4096 x 4096 x 8192: N(0,1) data
    quantised to e5m2 under E8M0 exponents U{-2..2} (bytes 125..129), bf16 out.
    Sampled rows against the oracle (bit-identical bf16 expected, 3e-2
    normalised bound asserted); all rows against the fp32 GPU product of the
    dequantised operands."""
    M = N = 4096
    K = 8192
    xa, xb, ea, eb = _mx_e5m2_inputs(M, N, K, seed=2002)
    qa = ops.quantize_mxe5m2(xa, ea)
    qb = ops.quantize_mxe5m2(xb, eb)
    del xa, xb
    ea_mc = ea.T.contiguous().T           # the reference's M-contiguous scale storage
    c = a8w8.matmul_scaled(qa, qb.T, ea_mc, eb)
    ops.check_status()
    assert c.dtype == torch.bfloat16
    rows = torch.randperm(M, generator=torch.Generator().manual_seed(2003))[:128].cuda()
    ref = mx.gemm_mxe5m2_ref(qa[rows].view(torch.uint8).cpu().numpy(),
                             qb.view(torch.uint8).cpu().numpy(),
                             ea[rows].cpu().numpy(), eb.cpu().numpy())
    got = bits16(c[rows])
    assert_close(mx.bf16_bits_to_f32(got), mx.bf16_bits_to_f32(ref), TOL_F8, ref_atol=False)
    print(f"cfg2 sampled rows bit-exact fraction {float(np.mean(got == ref)):.6f}")
    da = qa.float() * torch.exp2(ea.float() - 127).repeat_interleave(32, dim=1)
    db = qb.float() * torch.exp2(eb.float() - 127).repeat_interleave(32, dim=1)
    full = da @ db.T
    assert _gpu_normalised_err(c, full) <= TOL_F8


def test_a8w8_unscaled_full_size(cuda_device):
    """Unscaled e5m2 (the reference's a8w8 API, fp16 out) at 4096 x 4096 x 8192
    on the reference's own recipe (rand - 0.5, cast to e5m2): its
    allclose(atol=0.1) against the fp16-upcast torch product
    (kernels/gemm/intra_wave/a8w8/bench.py:133-142) and the normalised bound
    against the fp32 product; sampled rows against the oracle."""
    M = N = 4096
    K = 8192
    g = torch.Generator(device="cuda").manual_seed(2004)
    a = (torch.rand((M, K), generator=g, device="cuda").half() - 0.5).to(torch.float8_e5m2)
    b = (torch.rand((N, K), generator=g, device="cuda").half().T - 0.5).to(torch.float8_e5m2)
    c = a8w8.matmul(a, b)
    ops.check_status()
    assert c.dtype == torch.float16
    full = a.float() @ b.float()
    assert bool(torch.allclose(c.float(), full, atol=1e-1, rtol=0))
    assert _gpu_normalised_err(c, full) <= TOL_F8
    rows = torch.randperm(M, generator=torch.Generator().manual_seed(2005))[:128].cuda()
    ref = mx.gemm_e5m2_ref(a[rows].view(torch.uint8).cpu().numpy(),
                           b.T.contiguous().view(torch.uint8).cpu().numpy()).astype(np.float32)
    assert_close(as_f32(c[rows]), ref, TOL_F8)


def _decode_mxfp4_gpu(q: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    """Dequantise packed e2m1 + E8M0 on the GPU through the reference's own
    decode tables (kernels/gemm/intra_wave/a4w4/bench.py:80-112, committed as
    tests/golden/decode_tables.npz)."""
    t = golden("decode_tables.npz")
    nib = torch.from_numpy(t["mxfp4"].reshape(256, 2)[:16, 0].copy()).cuda()
    e8 = torch.from_numpy(t["e8m0"]).cuda()
    codes = torch.stack([q & 0xF, q >> 4], dim=-1).reshape(q.shape[0], -1).long()
    return nib[codes] * e8[s.long()].repeat_interleave(32, dim=1)


@pytest.mark.parametrize("K", [512, 1024, 2048, 4096, 8192, 16384, 32768])
@pytest.mark.parametrize("kind", ["fp16", "bf16", "bf8", "mxfp4"])
def test_reference_correctness_sweep_m4096(cuda_device, kind, K):
    """The reference benches' own correctness check (M = N = 4096, every K of
    their sweep, kernels/gemm/intra_wave/{a16w16,a8w8,a4w4}/bench.py
    test_correctness) on their input recipes: allclose(atol=0.1, rtol=0) and
    the normalised bound against the fp32 GPU product of the same operands."""
    M = N = 4096
    g = torch.Generator(device="cuda").manual_seed(K + len(kind))
    if kind in ("fp16", "bf16"):
        dt = torch.float16 if kind == "fp16" else torch.bfloat16
        a = torch.rand((M, K), generator=g, device="cuda").to(dt) - 0.5
        b = torch.rand((N, K), generator=g, device="cuda").to(dt).T - 0.5
        c = a16w16.matmul(a, b)
        full, tol = a.float() @ b.float(), TOL_F16
    elif kind == "bf8":
        a = (torch.rand((M, K), generator=g, device="cuda").half() - 0.5).to(torch.float8_e5m2)
        b = (torch.rand((N, K), generator=g, device="cuda").half().T - 0.5).to(torch.float8_e5m2)
        c = a8w8.matmul(a, b)
        full, tol = a.float() @ b.float(), TOL_F8
    else:
        a = torch.randint(0, 256, (M, K // 2), generator=g, device="cuda", dtype=torch.uint8)
        b = torch.randint(0, 256, (N, K // 2), generator=g, device="cuda", dtype=torch.uint8)
        sa = torch.randint(124, 128, (K // 32, M), generator=g, device="cuda",
                           dtype=torch.uint8).T
        sb = torch.randint(124, 128, (K // 32, N), generator=g, device="cuda",
                           dtype=torch.uint8).T
        c = a4w4.matmul(a, b, sa, sb)
        full, tol = _decode_mxfp4_gpu(a, sa) @ _decode_mxfp4_gpu(b, sb).T, TOL_F8
    ops.check_status()
    if kind == "mxfp4":
        # every product is a multiple of 2^-8 and every sum stays far inside
        # fp32's 24 bits, so the fp32 product is exact: bf16 bits must agree
        want = full.to(torch.bfloat16)
        assert torch.equal(c.view(torch.int16), want.view(torch.int16)), \
            f"{int((c != want).sum())} outputs differ from the exact sum rounded to bf16"
        # the reference checks against torch_reference, whose output is bf16
        full = want.float()
    # the reference's allclose(atol=0.1); bf16 outputs above 32 are spaced
    # wider than that, so bf16 also gets its rounding step (2^-8 relative)
    rtol = 2.0 ** -8 if kind == "bf16" else 0.0
    assert bool(torch.allclose(c.float(), full, atol=1e-1, rtol=rtol)), \
        f"max abs diff {(c.float() - full).abs().max().item():.3e}"
    assert _gpu_normalised_err(c, full) <= tol


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["fp16", "bf16"])
def test_a16w16_cfg1b_3840_sampled_rows(cuda_device, dtype):
    """Config-1's second case, 3840 x 3840 x 8192 (225 tiles of 256 x 256:
    3 full waves of 74 pairs and a 3-tile remainder): sampled rows against the
    oracle and all rows against the exact GPU product."""
    M = N = 3840
    K = 8192
    g = torch.Generator(device="cuda").manual_seed(38)
    a = (torch.randn((M, K), generator=g, device="cuda") / K ** 0.5).to(dtype)
    b_t = (torch.randn((N, K), generator=g, device="cuda") / K ** 0.5).to(dtype)
    c = a16w16.matmul(a, b_t.T)
    ops.check_status()
    rows = torch.randperm(M, generator=torch.Generator().manual_seed(39))[:192].cuda()
    if dtype == torch.float16:
        ref = mx.gemm_f16_ref(a[rows].cpu().numpy(), b_t.cpu().numpy()).astype(np.float32)
    else:
        ref = mx.bf16_bits_to_f32(mx.gemm_f16_ref(bits16(a[rows]), bits16(b_t), "bf16"))
    assert_close(as_f32(c[rows]), ref, TOL_F16, ref_atol=False)
    full = a.float() @ b_t.float().T
    assert ((c.float() - full).abs().max() / full.abs().max()).item() <= TOL_F16


def test_a4w4_cfg4_shard_sampled_blocks(cuda_device):
    """Config 4 at 8 GPUs: one rank's shard, 16384 x 6656 x 16384 MXFP4 from
    quantised N(0,1) data; eight seeded 128 x 128 blocks of C against the
    oracle's dequantise-then-matmul on just the rows and columns they need."""
    M, N, K = 16384, 53248 // 8, 16384
    g = torch.Generator(device="cuda").manual_seed(404)
    qa, sa = ops.quantize_mxfp4(torch.randn((M, K), generator=g, device="cuda"))
    qb, sb = ops.quantize_mxfp4(torch.randn((N, K), generator=g, device="cuda"))
    torch.cuda.empty_cache()
    c = a4w4.matmul(qa, qb, sa, sb)
    ops.check_status()
    pick = torch.Generator().manual_seed(405)
    for _ in range(8):
        r0 = int(torch.randint(0, M // 128, (1,), generator=pick)) * 128
        c0 = int(torch.randint(0, N // 128, (1,), generator=pick)) * 128
        ref = mx.gemm_mxfp4_ref(qa[r0:r0 + 128].cpu().numpy(), qb[c0:c0 + 128].cpu().numpy(),
                                sa[r0:r0 + 128].cpu().numpy(), sb[c0:c0 + 128].cpu().numpy())
        got = bits16(c[r0:r0 + 128, c0:c0 + 128])
        assert_close(mx.bf16_bits_to_f32(got), mx.bf16_bits_to_f32(ref), TOL_F8, ref_atol=False)


E5M2_SHAPES = [(128, 256, 128), (256, 512, 1024), (300, 700, 208), (1000, 1000, 2048)]


@pytest.mark.parametrize("shape", E5M2_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_a8w8_unscaled_matches_oracle(sched, shape):
    M, N, K = shape
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    a = (torch.rand((M, K), generator=g, device="cuda").half() - 0.5).to(torch.float8_e5m2)
    b = (torch.rand((N, K), generator=g, device="cuda").half().T - 0.5).to(torch.float8_e5m2)
    c = a8w8.matmul(a, b)
    ops.check_status()
    assert c.dtype == torch.float16
    ref = mx.gemm_e5m2_ref(a.view(torch.uint8).cpu().numpy(),
                           b.T.contiguous().view(torch.uint8).cpu().numpy()).astype(np.float32)
    assert_close(as_f32(c), ref, TOL_F8)


def test_a8w8_golden(cuda_device):
    g = golden("a8w8_e5m2_128x256x512.npz")
    a = torch.from_numpy(g["a"]).cuda().view(torch.float8_e5m2)
    b_t = torch.from_numpy(g["b_t"]).cuda().view(torch.float8_e5m2)
    c = a8w8.matmul(a, b_t.T)
    ops.check_status()
    assert_close(as_f32(c), g["c"].astype(np.float32), TOL_F8)


def _mx_e5m2_inputs(M, N, K, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    xa = torch.randn((M, K), generator=gen, device="cuda")
    xb = torch.randn((N, K), generator=gen, device="cuda")
    ea = torch.randint(125, 130, (M, K // 32), generator=gen, device="cuda").to(torch.uint8)
    eb = torch.randint(125, 130, (N, K // 32), generator=gen, device="cuda").to(torch.uint8)
    return xa, xb, ea, eb


@pytest.mark.parametrize("shape", [(128, 256, 128), (256, 512, 1024), (200, 300, 96),
                                   (1024, 768, 2048), (256, 384, 384)],
                         ids=lambda s: "x".join(map(str, s)))
def test_a8w8_scaled_matches_oracle(sched, shape):
    M, N, K = shape
    xa, xb, ea, eb = _mx_e5m2_inputs(M, N, K, M * N + K)
    qa = ops.quantize_mxe5m2(xa, ea)
    qb = ops.quantize_mxe5m2(xb, eb)
    # the reference-style M-contiguous storage for A's scales
    ea_mc = ea.T.contiguous().T
    c = a8w8.matmul_scaled(qa, qb.T, ea_mc, eb)
    ops.check_status()
    ref = mx.bf16_bits_to_f32(mx.gemm_mxe5m2_ref(
        qa.view(torch.uint8).cpu().numpy(), qb.view(torch.uint8).cpu().numpy(),
        ea.cpu().numpy(), eb.cpu().numpy()))
    assert_close(as_f32(c), ref, TOL_F8, ref_atol=False)


def _reference_style_mxfp4(M, N, K, seed):
    """Same recipe as the reference generator (kernels/gemm/intra_wave/a4w4/bench.py:115-146):
    random nibbles, scale bytes 124..127, A scales M-contiguous with M_pad rows."""
    g = torch.Generator().manual_seed(seed)
    a = (torch.randint(0, 16, (M, K // 2), generator=g, dtype=torch.uint8) << 4) | \
        torch.randint(0, 16, (M, K // 2), generator=g, dtype=torch.uint8)
    b = (torch.randint(0, 16, (N, K // 2), generator=g, dtype=torch.uint8) << 4) | \
        torch.randint(0, 16, (N, K // 2), generator=g, dtype=torch.uint8)
    m_pad = (M + 255) // 256 * 256
    sa = torch.randint(124, 128, (K // 32, m_pad), generator=g, dtype=torch.uint8).cuda().T[:M]
    sb = torch.randint(124, 128, (K // 32, N), generator=g, dtype=torch.uint8).cuda().T
    return a.cuda(), b.cuda(), sa, sb


@pytest.mark.parametrize("shape", [(128, 256, 256), (256, 512, 1024), (200, 320, 1024),
                                   (1000, 600, 2048), (128, 256, 64), (256, 512, 768),
                                   (200, 264, 1280)],
                         ids=lambda s: "x".join(map(str, s)))
def test_a4w4_reference_style_matches_oracle(sched, shape):
    M, N, K = shape
    a, b, sa, sb = _reference_style_mxfp4(M, N, K, M + 3 * N + K)
    c = a4w4.matmul(a, b, sa, sb)
    ops.check_status()
    ref_bits = mx.gemm_mxfp4_ref(a.cpu().numpy(), b.cpu().numpy(), sa.cpu().numpy(),
                                 sb.cpu().numpy())
    got_bits = bits16(c)
    assert_close(mx.bf16_bits_to_f32(got_bits), mx.bf16_bits_to_f32(ref_bits), TOL_F8)
    exact = float(np.mean(got_bits == ref_bits))
    print(f"mxfp4 {M}x{N}x{K}: bit-exact fraction {exact:.6f}")


@pytest.mark.parametrize("name", ["mxfp4_ref_128x256x256.npz", "mxfp4_ref_256x256x512.npz",
                                  "mxfp4_ref_200x320x1024.npz"])
def test_a4w4_golden(cuda_device, name):
    g = golden(name)
    a = torch.from_numpy(g["a"]).cuda()
    b = torch.from_numpy(g["b"]).cuda()
    sa = torch.from_numpy(g["a_scales"]).cuda()
    sb = torch.from_numpy(g["b_scales"]).cuda()
    c = a4w4.matmul(a, b, sa, sb)
    ops.check_status()
    got = bits16(c)
    assert_close(mx.bf16_bits_to_f32(got), mx.bf16_bits_to_f32(g["c_bf16"]), TOL_F8)


@pytest.mark.parametrize("shape", [(256, 256, 512), (512, 1024, 4096)],
                         ids=lambda s: "x".join(map(str, s)))
def test_a4w4_quantised_normal_inputs(sched, shape):
    """Config-3 recipe: N(0,1) data through the GPU quantiser, then the GEMM."""
    M, N, K = shape
    gen = torch.Generator(device="cuda").manual_seed(11)
    xa = torch.randn((M, K), generator=gen, device="cuda")
    xb = torch.randn((N, K), generator=gen, device="cuda")
    qa, sa = ops.quantize_mxfp4(xa)
    qb, sb = ops.quantize_mxfp4(xb)
    c = a4w4.matmul(qa, qb, sa, sb)
    ops.check_status()
    ref = mx.gemm_mxfp4_ref(qa.cpu().numpy(), qb.cpu().numpy(), sa.cpu().numpy(),
                            sb.cpu().numpy())
    assert_close(as_f32(c), mx.bf16_bits_to_f32(ref), TOL_F8, ref_atol=False)


def test_a4w4_full_size_sampled_rows(cuda_device):
    M = N = 4096
    K = 8192
    gen = torch.Generator(device="cuda").manual_seed(3)
    qa, sa = ops.quantize_mxfp4(torch.randn((M, K), generator=gen, device="cuda"))
    qb, sb = ops.quantize_mxfp4(torch.randn((N, K), generator=gen, device="cuda"))
    c = a4w4.matmul(qa, qb, sa, sb)
    ops.check_status()
    rows = torch.randperm(M, generator=torch.Generator().manual_seed(4))[:128].cuda()
    ref = mx.gemm_mxfp4_ref(qa[rows].cpu().numpy(), qb.cpu().numpy(),
                            sa[rows].cpu().numpy(), sb.cpu().numpy())
    assert_close(as_f32(c[rows]), mx.bf16_bits_to_f32(ref), TOL_F8, ref_atol=False)


def test_serpentine_k_order(cuda_device):
    """Odd waves walking K backwards change only the order of the fp32 sums:
    at 4096 x 4096 x 8192 (three full waves) FP16 stays within the tolerance of
    the fp32 product either way, and MXFP4 with the reference's inputs (whose
    products are multiples of 2^-8, summed exactly) is bit-identical."""
    M = N = 4096
    K = 8192
    a = (torch.randn((M, K), device="cuda") / K ** 0.5).half()
    b_t = (torch.randn((N, K), device="cuda") / K ** 0.5).half()
    qa, qb, sa, sb = _reference_style_mxfp4(M, N, K, seed=77)
    old = _lib.get_option(_lib.OPT_SERPENTINE)
    try:
        out = {}
        for serp in (1, 0):
            _lib.set_option(_lib.OPT_SERPENTINE, serp)
            out[serp] = (ops.gemm_f16(a, b_t), ops.gemm_mxf4(qa, qb, sa, sb))
        ops.check_status()
    finally:
        _lib.set_option(_lib.OPT_SERPENTINE, old)
    full = a.float() @ b_t.float().T
    for serp in (1, 0):
        assert _gpu_normalised_err(out[serp][0], full) <= TOL_F16
    assert torch.equal(out[1][1], out[0][1])


def test_banded_raster_fp16_8192(cuda_device):
    """A and B of 128 MiB each exceed L2, so the raster walks bands of 8 tile
    rows (32 MiB of A) column by column, with odd waves walking K backwards:
    the whole C against the fp32 GPU product."""
    M = N = K = 8192
    assert ops.plan(_lib.KIND_F16, M, N, K, torch.cuda.get_device_properties(0)
                    .multi_processor_count)["group_m"] == 8
    g = torch.Generator(device="cuda").manual_seed(88)
    a = (torch.randn((M, K), generator=g, device="cuda") / K ** 0.5).half()
    b_t = (torch.randn((N, K), generator=g, device="cuda") / K ** 0.5).half()
    c = ops.gemm_f16(a, b_t)
    ops.check_status()
    assert _gpu_normalised_err(c, a.float() @ b_t.float().T) <= TOL_F16


def test_repeated_calls_are_deterministic(cuda_device):
    """Stream-K reduces partials in a fixed order: identical inputs, identical bits."""
    old = _lib.get_option(_lib.OPT_MIN_SK_ITERS)
    _lib.set_option(_lib.OPT_MIN_SK_ITERS, 1)
    try:
        a = torch.randn((512, 4096), device="cuda", dtype=torch.bfloat16)
        b_t = torch.randn((512, 4096), device="cuda", dtype=torch.bfloat16)
        c0 = ops.gemm_f16(a, b_t)
        for _ in range(3):
            assert torch.equal(ops.gemm_f16(a, b_t), c0)
        ops.check_status()
    finally:
        _lib.set_option(_lib.OPT_MIN_SK_ITERS, old)


@pytest.mark.parametrize("layout", ["m_contig", "k_contig", "strided", "odd_k"])
@pytest.mark.parametrize("pair", [1, 0])
def test_a4w4_scale_layouts(cuda_device, layout, pair):
    """Scales of any strides: row-contiguous (the reference's storage), K-contiguous,
    a strided view, and a K/32 that is not a multiple of 4 (byte gathers)."""
    M, N, K = (300, 520, 1024) if layout != "odd_k" else (256, 384, 192)
    a, b, sa, sb = _reference_style_mxfp4(M, N, K, 17)
    if layout == "k_contig":
        sa, sb = sa.contiguous(), sb.contiguous()
    elif layout == "strided":
        big_a = torch.full((M, 2 * (K // 32)), 255, dtype=torch.uint8, device="cuda")
        big_b = torch.full((N, 2 * (K // 32)), 255, dtype=torch.uint8, device="cuda")
        big_a[:, ::2] = sa
        big_b[:, ::2] = sb
        sa, sb = big_a[:, ::2], big_b[:, ::2]
    elif layout == "odd_k":
        sa = sa.contiguous()
    old = _lib.get_option(_lib.OPT_PAIR)
    _lib.set_option(_lib.OPT_PAIR, pair)
    try:
        c = a4w4.matmul(a, b, sa, sb)
        ops.check_status()
    finally:
        _lib.set_option(_lib.OPT_PAIR, old)
    ref = mx.gemm_mxfp4_ref(a.cpu().numpy(), b.cpu().numpy(), sa.cpu().numpy(), sb.cpu().numpy())
    assert_close(as_f32(c), mx.bf16_bits_to_f32(ref), TOL_F8)


@pytest.mark.parametrize("kind", ["mxfp4", "mxe5m2"])
def test_preblocked_scales_match_per_call_relayout(cuda_device, kind):
    """Scales converted once with block_scales give bit-identical results to
    scales relaid on every call."""
    M, N, K = 384, 640, 1536
    if kind == "mxfp4":
        a, b, sa, sb = _reference_style_mxfp4(M, N, K, 23)
        c0 = a4w4.matmul(a, b, sa, sb)
        c1 = a4w4.matmul(a, b, ops.block_scales(sa), ops.block_scales(sb))
    else:
        xa, xb, ea, eb = _mx_e5m2_inputs(M, N, K, 29)
        qa, qb = ops.quantize_mxe5m2(xa, ea), ops.quantize_mxe5m2(xb, eb)
        c0 = ops.gemm_f8(qa, qb, a_scales=ea, b_scales=eb, out_dtype=torch.bfloat16)
        c1 = ops.gemm_f8(qa, qb, a_scales=ops.block_scales(ea), b_scales=eb,
                         out_dtype=torch.bfloat16)
    ops.check_status()
    assert torch.equal(c0, c1)


# ------------------------------------------------------------- small M (swap-AB)
SKINNY_SHAPES = [(1, 256, 64), (7, 1000, 136), (16, 4096, 1024), (33, 300, 2048),
                 (64, 520, 4096), (100, 2048, 512), (128, 384, 8192), (5, 129, 40000)]


@pytest.fixture
def skinny_on(cuda_device):
    old = _lib.get_option(_lib.OPT_SKINNY_MAX_M)
    _lib.set_option(_lib.OPT_SKINNY_MAX_M, 128)
    yield
    _lib.set_option(_lib.OPT_SKINNY_MAX_M, old)
    ops.check_status(cuda_device)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["fp16", "bf16"])
@pytest.mark.parametrize("shape", SKINNY_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_skinny_a16w16_matches_oracle(skinny_on, dtype, shape):
    M, N, K = shape
    g = torch.Generator(device="cuda").manual_seed(M * 5 + N + K)
    a = torch.rand((M, K), generator=g, device="cuda", dtype=torch.float32).to(dtype) - 0.5
    b_t = torch.rand((N, K), generator=g, device="cuda", dtype=torch.float32).to(dtype) - 0.5
    c = a16w16.matmul(a, b_t.T)
    ops.check_status()
    if dtype == torch.float16:
        ref = mx.gemm_f16_ref(a.cpu().numpy(), b_t.cpu().numpy(), "f16").astype(np.float32)
    else:
        ref = mx.bf16_bits_to_f32(mx.gemm_f16_ref(bits16(a), bits16(b_t), "bf16"))
    assert_close(as_f32(c), ref, TOL_F16)


@pytest.mark.parametrize("shape", [(1, 512, 1024), (48, 1000, 2048), (128, 256, 8192)],
                         ids=lambda s: "x".join(map(str, s)))
def test_skinny_a8w8_matches_oracle(skinny_on, shape):
    M, N, K = shape
    g = torch.Generator(device="cuda").manual_seed(M + 3 * N + K)
    a = (torch.rand((M, K), generator=g, device="cuda").half() - 0.5).to(torch.float8_e5m2)
    b_t = (torch.rand((N, K), generator=g, device="cuda").half() - 0.5).to(torch.float8_e5m2)
    c = a8w8.matmul(a, b_t.T)
    ops.check_status()
    ref = mx.gemm_e5m2_ref(a.view(torch.uint8).cpu().numpy(),
                           b_t.view(torch.uint8).cpu().numpy()).astype(np.float32)
    assert_close(as_f32(c), ref, TOL_F8)


def test_skinny_split_reduction_is_deterministic(skinny_on):
    """Several K splits per tile add their partials in split order: repeated
    calls give bit-identical C."""
    g = torch.Generator(device="cuda").manual_seed(21)
    a = torch.randn((16, 8192), generator=g, device="cuda").half()
    b_t = torch.randn((2048, 8192), generator=g, device="cuda").half()
    first = ops.gemm_f16(a, b_t)
    for _ in range(5):
        assert torch.equal(ops.gemm_f16(a, b_t), first)
    ops.check_status()


def test_skinny_agrees_with_the_persistent_kernel(cuda_device):
    g = torch.Generator(device="cuda").manual_seed(8)
    a = torch.randn((64, 4096), generator=g, device="cuda").half() / 64
    b_t = torch.randn((3000, 4096), generator=g, device="cuda").half() / 64
    old = _lib.get_option(_lib.OPT_SKINNY_MAX_M)
    try:
        _lib.set_option(_lib.OPT_SKINNY_MAX_M, 128)
        c_skinny = ops.gemm_f16(a, b_t)
        _lib.set_option(_lib.OPT_SKINNY_MAX_M, 0)
        c_main = ops.gemm_f16(a, b_t)
    finally:
        _lib.set_option(_lib.OPT_SKINNY_MAX_M, old)
    ops.check_status()
    assert_close(as_f32(c_skinny), as_f32(c_main), TOL_F16, ref_atol=False)


def test_small_m_wider_than_the_counter_region(skinny_on):
    """The small-M kernel keeps one arrival counter per 128-column tile in the
    workspace's flag region (four words per SM); a problem with more tiles than
    that takes the persistent kernel and is still correct."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    M, N, K = 8, sms * 4 * 128 + 256, 128
    g = torch.Generator(device="cuda").manual_seed(31)
    a = torch.rand((M, K), generator=g, device="cuda").half() - 0.5
    b_t = torch.rand((N, K), generator=g, device="cuda").half() - 0.5
    c = ops.gemm_f16(a, b_t)
    ops.check_status()
    ref = a.float() @ b_t.float().T
    assert_close(as_f32(c), ref.cpu().numpy(), TOL_F16)


def test_flag_region_stays_zero_across_mixed_calls(cuda_device):
    """One workspace shared by calls of different kinds and geometries: the
    flag words at its start are zero after every call (unsplit scaled GEMMs,
    split GEMMs and small-M GEMMs all keep their data after the region)."""
    lib = _lib.lib()
    sms = torch.cuda.get_device_properties(cuda_device).multi_processor_count
    flag_bytes = (sms * 16 + 255) // 256 * 256
    ws = torch.zeros(256 << 20, dtype=torch.uint8, device=cuda_device)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    stream = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device="cuda").manual_seed(4)

    def f16(M, N, K):
        a = torch.randn((M, K), generator=g, device="cuda").half() / 32
        b = torch.randn((N, K), generator=g, device="cuda").half() / 32
        c = torch.empty((M, N), dtype=torch.half, device="cuda")
        assert lib.b2g_gemm_f16(a.data_ptr(), K, b.data_ptr(), K, c.data_ptr(), N, M, N, K, 0, 0,
                                ws.data_ptr(), ws.numel(), status.data_ptr(), stream) == 0
        return c, (a.float() @ b.float().T)

    def fp4(M, N, K):
        qa, sa = ops.quantize_mxfp4(torch.randn((M, K), generator=g, device="cuda"))
        qb, sb = ops.quantize_mxfp4(torch.randn((N, K), generator=g, device="cuda"))
        c = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
        assert lib.b2g_gemm_mxf4(qa.data_ptr(), K // 2, qb.data_ptr(), K // 2, sa.data_ptr(),
                                 sa.stride(0), sa.stride(1), sb.data_ptr(), sb.stride(0),
                                 sb.stride(1), c.data_ptr(), N, M, N, K, 1, ws.data_ptr(),
                                 ws.numel(), status.data_ptr(), stream) == 0

    for step in (lambda: fp4(8192, 8192, 1024),      # no split tiles: scales relaid out
                 lambda: f16(4096, 4096, 2048),      # split tiles: flags used
                 lambda: f16(16, 4096, 8192),        # small M: split counters
                 lambda: fp4(4096, 4096, 2048)):
        out = step()
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert int(ws[:flag_bytes].count_nonzero().item()) == 0
        if out is not None:
            c, ref = out
            assert_close(as_f32(c), ref.cpu().numpy(), TOL_F16, ref_atol=False)


# --------------------------------------------------- MoE grouped MXFP4 GEMM
def _grouped_inputs(sizes, N, K, seed, tile=256):
    """Tokens sorted by expert, each expert's segment padded to `tile` rows;
    reference-style random nibbles and E8M0 bytes 124..127, A scales
    M-contiguous (the reference's storage)."""
    g = torch.Generator().manual_seed(seed)
    padded = [(s + tile - 1) // tile * tile for s in sizes]
    offsets = np.concatenate([[0], np.cumsum(padded)]).astype(np.int32)
    M, E = int(offsets[-1]), len(sizes)
    a = torch.randint(0, 256, (M, K // 2), generator=g, dtype=torch.uint8)
    b = torch.randint(0, 256, (E * N, K // 2), generator=g, dtype=torch.uint8)
    sa = torch.randint(124, 128, (K // 32, M), generator=g, dtype=torch.uint8).T
    sb = torch.randint(124, 128, (E * N, K // 32), generator=g, dtype=torch.uint8)
    return a, b, sa, sb, offsets


@pytest.mark.parametrize("sizes,N,K", [([300, 0, 512, 40], 512, 1024), ([256] * 8, 256, 512),
                                       ([1000, 17], 384, 2048), ([0, 0, 600], 1024, 768)],
                         ids=["ragged", "uniform8", "two", "leading_empty"])
@pytest.mark.parametrize("pair", [1, 0])
def test_grouped_mxfp4_matches_oracle(cuda_device, sizes, N, K, pair):
    tile = 256 if pair else 128
    a, b, sa, sb, offsets = _grouped_inputs(sizes, N, K, sum(sizes) + N + K, tile)
    ref = mx.gemm_mxfp4_grouped_ref(a.numpy(), b.numpy(), sa.numpy(), sb.numpy(), offsets)
    old = _lib.get_option(_lib.OPT_PAIR)
    try:
        _lib.set_option(_lib.OPT_PAIR, pair)
        c = a4w4.grouped_matmul(a.cuda(), b.cuda(), sa.cuda(), sb.cuda(),
                                torch.from_numpy(offsets).cuda())
        ops.check_status()
    finally:
        _lib.set_option(_lib.OPT_PAIR, old)
    got = bits16(c)
    assert_close(mx.bf16_bits_to_f32(got), mx.bf16_bits_to_f32(ref), TOL_F8)
    print(f"grouped {sizes}: bit-exact fraction {float(np.mean(got == ref)):.6f}")


def test_grouped_mxfp4_preblocked_expert_scales_and_3d_weights(cuda_device):
    """Static expert weights: scales relaid once (BlockedScales) and weights
    passed as (E, N, K/2) give the same C as the per-call path."""
    a, b, sa, sb, offsets = _grouped_inputs([512, 256, 768], 256, 1024, 77)
    offs = torch.from_numpy(offsets).cuda()
    E = len(offsets) - 1
    c1 = a4w4.grouped_matmul(a.cuda(), b.cuda(), sa.cuda(), sb.cuda(), offs)
    sb_blocked = ops.block_scales(sb.cuda(), 1024)
    c2 = a4w4.grouped_matmul(a.cuda(), b.cuda().view(E, 256, -1), sa.cuda(), sb_blocked, offs)
    ops.check_status()
    assert torch.equal(c1, c2)


def test_grouped_mxfp4_rejects_bad_offsets(cuda_device):
    """Offsets that are not multiples of the tile height: status code, nothing
    written; the next valid call works."""
    a, b, sa, sb, offsets = _grouped_inputs([256, 256], 256, 512, 5)
    bad = offsets.copy()
    bad[1] = 200
    c = torch.full((int(offsets[-1]), 256), 7.0, dtype=torch.bfloat16, device="cuda")
    a4w4.grouped_matmul(a.cuda(), b.cuda(), sa.cuda(), sb.cuda(), torch.from_numpy(bad).cuda(),
                        c=c)
    with pytest.raises(_lib.B2GError) as info:
        ops.check_status()
    assert info.value.code == _lib.STATUS_BAD_GROUPS
    assert bool((c == 7.0).all())
    c_ok = a4w4.grouped_matmul(a.cuda(), b.cuda(), sa.cuda(), sb.cuda(),
                               torch.from_numpy(offsets).cuda())
    ops.check_status()
    ref = mx.gemm_mxfp4_grouped_ref(a.numpy(), b.numpy(), sa.numpy(), sb.numpy(), offsets)
    assert_close(as_f32(c_ok), mx.bf16_bits_to_f32(ref), TOL_F8)
