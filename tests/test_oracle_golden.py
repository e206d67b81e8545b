"""Pins the CPU oracle (oracle/mx.py) to golden vectors made by the reference's
own functions (tests/golden/make_golden.py) - no GPU needed."""

from __future__ import annotations

import numpy as np
import pytest
from conftest import golden

from oracle import mx


def test_decode_tables_match_reference():
    g = golden("decode_tables.npz")
    b = g["bytes"].reshape(1, 256)
    np.testing.assert_array_equal(mx.mxfp4_to_f32(b)[0].view(np.uint32),
                                  g["mxfp4"].view(np.uint32))  # incl. the sign of -0
    e = mx.e8m0_to_f32(g["bytes"])
    ref = g["e8m0"]
    assert np.isnan(e[255]) and np.isnan(ref[255])
    np.testing.assert_array_equal(e[:255], ref[:255])


@pytest.mark.parametrize("name", ["mxfp4_ref_128x256x256.npz", "mxfp4_ref_256x256x512.npz",
                                  "mxfp4_ref_200x320x1024.npz"])
def test_mxfp4_gemm_oracle_matches_reference(name):
    g = golden(name)
    c = mx.gemm_mxfp4_ref(g["a"], g["b"], g["a_scales"], g["b_scales"])
    # reference-style inputs: every product is a multiple of 2^-8 and the fp32
    # sums are exact, so the bf16 result is bit-identical whatever the order
    np.testing.assert_array_equal(c, g["c_bf16"])


def test_mxfp4_reference_scale_layout_is_m_contiguous():
    g = golden("mxfp4_ref_200x320x1024.npz")
    # torch.randint((K//32, M_pad)).T[:M] -> strides (1, M_pad), M_pad = 256
    assert tuple(g["a_scales_strides"]) == (1, 256)


@pytest.mark.parametrize("name,out", [("a16w16_f16_128x256x320.npz", "f16"),
                                      ("a16w16_bf16_128x256x320.npz", "bf16")])
def test_a16w16_oracle_close_to_reference(name, out):
    g = golden(name)
    c = mx.gemm_f16_ref(g["a"], g["b_t"], out=out)
    if out == "f16":
        ref, got = g["c"].astype(np.float32), c.astype(np.float32)
    else:
        ref, got = mx.bf16_bits_to_f32(g["c"]), mx.bf16_bits_to_f32(c)
    # same math, different fp32 summation order than torch's CPU kernel
    assert mx.normalised_max_abs(got, ref) <= 1e-2
    assert np.allclose(got, ref, atol=1e-1, rtol=0)


def test_a8w8_oracle_matches_reference():
    g = golden("a8w8_e5m2_128x256x512.npz")
    c = mx.gemm_e5m2_ref(g["a"], g["b_t"]).astype(np.float32)
    ref = g["c"].astype(np.float32)
    assert mx.normalised_max_abs(c, ref) <= 1e-3
    assert np.allclose(c, ref, atol=1e-1, rtol=0)


def test_e5m2_rounding_matches_torch_cast():
    g = golden("e5m2_cast.npz")
    q = mx.f32_to_e5m2(g["x"])
    np.testing.assert_array_equal(q, g["q"])


def test_e5m2_decode_roundtrip():
    allb = np.arange(256, dtype=np.uint8)
    v = mx.e5m2_to_f32(allb)
    fin = np.isfinite(v)
    np.testing.assert_array_equal(mx.f32_to_e5m2(v[fin]), allb[fin])
