"""Quantise-and-pack kernels on a B200, bit-exact against the CPU oracle and
against torch's own float8_e5m2 cast (golden vectors)."""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import golden

from gfx950_gluon_tutorials_b200 import ops
from oracle import mx

pytestmark = pytest.mark.gpu


def _edge_matrix(rows: int, K: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, K)).astype(np.float32)
    x[0, :32] = 0.0                                   # all-zero block
    x[0, 32:64] = -0.0                                # all negative-zero block
    x[1, :32] = np.nan if K >= 32 else 0              # NaN block
    x[1, 40] = np.inf                                 # inf block
    x[2, :32] = np.ldexp(1.0, -140) * rng.uniform(-1, 1, 32)   # subnormal block
    x[3, :32] = np.float32(3.0e38) * rng.uniform(-1, 1, 32)    # near FLT_MAX
    # e2m1 ties after scaling: amax 4 -> s = 0, so the values below are the ties
    x[4, :32] = np.resize(np.array([4.0, .25, .75, 1.25, 1.75, 2.5, 3.5, 5.0, -0.25, -5.0],
                                   np.float32), 32)
    x[5, :32] = np.resize(np.array([6.0, 7.0, 7.99, -7.5, 0.1, -0.1], np.float32), 32)
    return x


@pytest.mark.parametrize("rows,K", [(64, 256), (300, 1024), (1024, 4096)])
def test_quantize_mxfp4_bit_exact(cuda_device, rows, K):
    x = _edge_matrix(rows, K, rows + K)
    q, s = ops.quantize_mxfp4(torch.from_numpy(x).cuda(), rows_pad=(rows + 255) // 256 * 256)
    assert s.stride() == (1, (rows + 255) // 256 * 256)  # reference storage
    q_ref, s_ref = mx.quantize_mxfp4(x)
    np.testing.assert_array_equal(s.cpu().numpy(), s_ref)
    np.testing.assert_array_equal(q.cpu().numpy(), q_ref)


def test_quantize_mxfp4_roundtrip_error_bound(cuda_device):
    """Decoding a quantised block reproduces each value to within half an e2m1
    step of the block scale (size-independent property)."""
    x = torch.randn((512, 2048), device="cuda")
    q, s = ops.quantize_mxfp4(x)
    deq = mx.mxfp4_to_f32(q.cpu().numpy()) * np.repeat(mx.e8m0_to_f32(s.cpu().numpy()), 32, 1)
    xs = x.cpu().numpy()
    scale = np.repeat(mx.e8m0_to_f32(s.cpu().numpy()), 32, 1)
    # the largest step of the e2m1 grid is 2 (between 4 and 6): half-step 1 * scale,
    # plus saturation for |x|/scale in (6, 8): error below 2 * scale
    assert np.all(np.abs(deq - xs) <= 2.0 * scale + 1e-30)


@pytest.mark.parametrize("rows,K", [(64, 256), (300, 1024)])
def test_quantize_mxe5m2_bit_exact(cuda_device, rows, K):
    x = _edge_matrix(rows, K, 7 * rows + K)
    rng = np.random.default_rng(rows)
    e = rng.integers(125, 130, (rows, K // 32)).astype(np.uint8)
    e[6, 0] = 255
    e[7, 0] = 254
    e[8, 0] = 0
    q = ops.quantize_mxe5m2(torch.from_numpy(x).cuda(), torch.from_numpy(e).cuda())
    q_ref = mx.quantize_mxe5m2(x, e)
    np.testing.assert_array_equal(q.view(torch.uint8).cpu().numpy(), q_ref)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_cast_e5m2_matches_torch(cuda_device, dtype):
    g = golden("e5m2_cast.npz")
    x = torch.from_numpy(g["x"]).cuda().to(dtype)
    got = ops.cast_e5m2(x).view(torch.uint8).cpu().numpy()
    # torch's own cast of the same (possibly narrowed) values
    want = x.float().cpu().to(torch.float8_e5m2).view(torch.uint8).numpy()
    np.testing.assert_array_equal(got, want)
    if dtype == torch.float32:
        np.testing.assert_array_equal(got, g["q"])


def _check_nearest_e2m1(x: torch.Tensor, q: torch.Tensor, s: torch.Tensor) -> None:
    """Every code the quantiser emitted, decoded through the reference's decode
    tables (kernels/gemm/intra_wave/a4w4/bench.py:80-112, committed as
    tests/golden/decode_tables.npz) and multiplied by its block's E8M0 scale,
    is the grid value nearest to x / scale, with ties to the even code and
    magnitudes above 6 saturated to 6. Scales follow the OCP MX rule
    s = floor(log2(max|x|)) - 2 (byte s + 127, at least 0; an all-zero block
    byte 0; a non-finite block byte 255 with zero codes)."""
    t = golden("decode_tables.npz")
    nib = torch.from_numpy(t["mxfp4"].reshape(256, 2)[:16, 0].copy()).cuda().double()
    e8 = torch.from_numpy(t["e8m0"]).cuda().double()
    mags = nib[:8]                                         # 0, .5, 1, 1.5, 2, 3, 4, 6
    rows, K = x.shape
    for r0 in range(0, rows, 256):
        xb = x[r0:r0 + 256].double()
        qb = q[r0:r0 + 256]
        codes = torch.stack([qb & 0xF, qb >> 4], dim=-1).reshape(xb.shape[0], K).long()
        sb = s[r0:r0 + 256].long()
        blocks = xb.reshape(xb.shape[0], K // 32, 32)
        finite = torch.isfinite(blocks).all(dim=2)
        amax = blocks.abs().amax(dim=2)
        # scale byte from the block max (finite blocks)
        want_s = torch.where(amax > 0, torch.floor(torch.log2(amax)) - 2 + 127,
                             torch.zeros_like(amax)).clamp(min=0)
        want_s = torch.where(finite, want_s, torch.full_like(amax, 255))
        assert torch.equal(sb, want_s.long()), "scale byte differs from the OCP MX rule"
        assert bool((codes.reshape_as(blocks)[~finite] == 0).all()), "non-finite block codes"
        scale = e8[sb].repeat_interleave(32, dim=1)
        ok = finite.repeat_interleave(32, dim=1)
        y = torch.where(ok, xb / torch.where(ok, scale, torch.ones_like(scale)),
                        torch.zeros_like(xb))
        dist = (y.abs().unsqueeze(-1) - mags).abs()            # (r, K, 8)
        best = dist.min(dim=-1).values
        got_mag = nib[codes & 7]
        got_d = (y.abs() - got_mag).abs()
        assert bool((got_d[ok] == best[ok]).all()), "a code is not the nearest grid value"
        ties = (dist == best.unsqueeze(-1)).sum(dim=-1) > 1
        assert bool(((codes & 1)[ok & ties] == 0).all()), "a tie did not round to the even code"
        nz = ok & (got_mag > 0)
        assert bool(((codes >> 3)[nz] == (y[nz] < 0).long()).all()), "sign bit"


def test_quantize_mxfp4_nearest_grid_value_cfg3(cuda_device):
    """BASELINE config-3 operands (4096 x 8192 N(0,1)) through the GPU quantiser,
    pinned to the reference's decode table element by element."""
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn((4096, 8192), generator=g, device="cuda")
    q, s = ops.quantize_mxfp4(x, rows_pad=4096)
    _check_nearest_e2m1(x, q, s)


def test_quantize_mxfp4_nearest_grid_value_edges(cuda_device):
    """The edge matrix (zero, negative-zero, NaN, inf, subnormal, near-FLT_MAX
    and exact-tie blocks) pinned the same way."""
    x = torch.from_numpy(_edge_matrix(1024, 4096, 99)).cuda()
    q, s = ops.quantize_mxfp4(x)
    _check_nearest_e2m1(x, q, s)


def _blocked_ref(s: np.ndarray) -> np.ndarray:
    """The GEMM's blocked scale layout restated in numpy: for 128-row block rb
    and 4-scale group g, 512 bytes at (rb * groups + g) * 512 whose byte
    r0 * 16 + r1 * 4 + j is the scale of row 128 rb + 32 r1 + r0, k-block
    4 g + j; rows and k-blocks past the matrix hold 127."""
    rows, kb = s.shape
    rbs, groups = (rows + 127) // 128, (kb + 3) // 4
    full = np.full((rbs * 128, groups * 4), 127, np.uint8)
    full[:rows, :kb] = s
    # (rb, r1, r0, g, j) -> (rb, g, r0, r1, j)
    t = full.reshape(rbs, 4, 32, groups, 4).transpose(0, 3, 2, 1, 4)
    return np.ascontiguousarray(t).reshape(-1)


@pytest.mark.parametrize("layout", ["k_contig", "k_contig_ragged", "k_contig_padded_rows",
                                    "m_contig", "m_contig_rows_pad", "strided"])
@pytest.mark.parametrize("rows,K", [(4096, 8192), (300, 8192), (300, 2080), (128, 32),
                                    (1, 4096)])
def test_block_scales_layout(cuda_device, layout, rows, K):
    """The relayout (its coalesced K-contiguous path and its generic path)
    against the layout restated in numpy, byte for byte."""
    kb = K // 32
    g = torch.Generator(device="cuda").manual_seed(rows * 3 + kb)
    base = torch.randint(0, 255, (rows, kb), generator=g, device="cuda").to(torch.uint8)
    if layout == "k_contig":
        s = base
    elif layout == "k_contig_ragged":
        s = base[:, : max(kb - 3, 1)]          # K/32 not a multiple of 16 (or of 4)
    elif layout == "k_contig_padded_rows":
        store = torch.zeros((rows, kb + 16), dtype=torch.uint8, device="cuda")
        store[:, :kb] = base
        s = store[:, :kb]                      # row stride kb + 16 (16-byte aligned)
    elif layout == "m_contig":
        s = base.T.contiguous().T
    elif layout == "m_contig_rows_pad":
        # the reference's storage: strides (1, rows rounded up to 256)
        rows_pad = (rows + 255) // 256 * 256
        store = torch.zeros((kb, rows_pad), dtype=torch.uint8, device="cuda")
        store[:, :rows] = base.T
        s = store[:, :rows].T
    else:
        store = torch.zeros((rows, 2 * kb + 1), dtype=torch.uint8, device="cuda")
        store[:, : 2 * kb : 2] = base
        s = store[:, : 2 * kb : 2]             # k stride 2, odd row stride
    blocked = ops.block_scales(s)
    torch.cuda.synchronize()
    ops.check_status()
    np.testing.assert_array_equal(blocked.data.cpu().numpy(), _blocked_ref(s.cpu().numpy()))
