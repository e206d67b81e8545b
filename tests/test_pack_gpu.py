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
