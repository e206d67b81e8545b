"""Attention forward, CPU side: the oracle against the reference's golden
vectors, the reference's tolerance rule, the host helpers of the drop-in
module and the C-ABI argument checks (which run before any device call)."""

from __future__ import annotations

import ctypes
import glob
import os

import numpy as np
import pytest
import torch

from gfx950_gluon_tutorials_b200 import _lib, attention
from oracle import attention as oa

GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "attention_*.npz")))


def load_golden(path):
    """(q, k, v as float32 bhsd, o_ref, dims, dtype name, sm_scale) of one fixture."""
    z = np.load(path)
    name = str(z["dtype"])
    tdt = torch.float16 if name == "float16" else torch.bfloat16
    as_f32 = [torch.from_numpy(z[n].view(np.int16)).view(tdt).float().numpy() for n in "qkv"]
    return (*as_f32, z["o_ref"], tuple(int(x) for x in z["dims"]), name, float(z["sm_scale"]))


def test_golden_fixtures_present():
    assert len(GOLDEN) >= 4


@pytest.mark.parametrize("path", GOLDEN, ids=lambda p: os.path.basename(p)[:-4])
def test_oracle_matches_reference_sdpa(path):
    q, k, v, o_ref, dims, _, sm_scale = load_golden(path)
    o, lse = oa.sdpa_ref(q, k, v, sm_scale)
    assert o.shape == o_ref.shape
    # fp32 (reference) against float64 (oracle): a few fp32 ULPs of the output
    np.testing.assert_allclose(o, o_ref, rtol=1e-5, atol=2e-6)
    B, HQ, HK, Sq, Sk, D = dims
    assert lse.shape == (B, HQ, Sq)


def test_oracle_lse_is_logsumexp():
    rng = np.random.default_rng(3)
    q = rng.standard_normal((1, 2, 5, 64))
    k = rng.standard_normal((1, 1, 7, 64))
    v = rng.standard_normal((1, 1, 7, 64))
    o, lse = oa.sdpa_ref(q, k, v, 0.125)
    s = np.einsum("bhmd,bhnd->bhmn", q, np.repeat(k, 2, axis=1)) * 0.125
    np.testing.assert_allclose(lse, np.log(np.exp(s).sum(-1)), rtol=1e-12)
    p = np.exp(s - lse[..., None])
    np.testing.assert_allclose(o, p @ np.repeat(v, 2, axis=1), rtol=1e-12)


def test_oracle_gqa_repeats_heads_in_groups():
    """Query head h reads key/value head h // (HQ // HK) (repeat_interleave)."""
    rng = np.random.default_rng(4)
    q = rng.standard_normal((1, 4, 3, 64))
    k = rng.standard_normal((1, 2, 6, 64))
    v = rng.standard_normal((1, 2, 6, 64))
    o, _ = oa.sdpa_ref(q, k, v, 0.1)
    for h in range(4):
        oh, _ = oa.sdpa_ref(q[:, h:h + 1], k[:, h // 2:h // 2 + 1], v[:, h // 2:h // 2 + 1], 0.1)
        np.testing.assert_allclose(o[:, h:h + 1], oh, rtol=1e-13)


def test_check_output_floor_scales_with_reference():
    ref = np.full((4, 4), 8.0)
    # two bf16 ULPs at magnitude 8 is 0.125: 0.1 off passes, 0.2 off fails
    assert oa.check_output(ref + 0.1, ref, "bfloat16")[0]
    assert not oa.check_output(ref + 0.2, ref, "bfloat16")[0]
    small = np.full((4, 4), 1e-4)
    assert oa.check_output(small + 9e-4, small, "float16")[0]
    assert not oa.check_output(small + 2e-3, small, "float16")[0]
    bad = ref.copy()
    bad[0, 0] = np.nan
    assert not oa.check_output(bad, ref, "bfloat16")[0]


def test_check_output_catches_planted_softmax_error():
    """A softmax that forgets the GQA grouping (planted in the oracle's inputs)
    is far outside the tolerance."""
    q, k, v, o_ref, _, name, sm_scale = load_golden(
        [p for p in GOLDEN if "h4k2" in p][0])
    wrong_k = np.concatenate([k[:, :1]] * k.shape[1], axis=1)  # every head reads group 0
    o_bad, _ = oa.sdpa_ref(q, wrong_k, v, sm_scale)
    assert not oa.check_output(o_bad, o_ref, name)[0]


# ------------------------------------------------------------ host helpers --
def test_shape_and_strides_from_layout():
    md = attention.MetaData(sm_scale=0.1)
    md.layout = "bhsd"
    q = torch.empty(2, 8, 100, 64)
    k = torch.empty(2, 2, 100, 64)
    assert attention.get_shape_from_layout(q, k, md) == (2, 8, 2, 64)
    strides = attention.get_strides_from_layout(q, k, k, q, md)
    assert strides[0] == q.stride()
    md.layout = "bshd"
    q = torch.empty(2, 100, 8, 64)
    k = torch.empty(2, 100, 2, 64)
    assert attention.get_shape_from_layout(q, k, md) == (2, 8, 2, 64)
    qs = attention.get_strides_from_layout(q, k, k, q, md)[0]
    assert qs == (q.stride(0), q.stride(2), q.stride(1), q.stride(3))
    md.layout = "sbhd"
    with pytest.raises(ValueError):
        attention.get_shape_from_layout(q, k, md)


def test_compute_flops():
    assert attention.compute_flops(1, 64, 8192, 8192, 128, False) == 4 * 64 * 8192 ** 2 * 128
    # causal with M == N counts the lower triangle with its diagonal
    assert attention.compute_flops(1, 1, 4, 4, 2, True) == 2 * 2.0 * (16 - 6) * 2


def test_input_helper_cpu_recipe():
    q, k, v, md = attention.input_helper(1, 4, 2, 64, 96, 64, torch.float32, "bshd", device="cpu")
    assert q.shape == (1, 64, 4, 64) and k.shape == (1, 96, 2, 64) and v.shape == k.shape
    assert md.layout == "bshd" and md.max_seqlens_q == 64 and md.max_seqlens_k == 96
    assert md.sm_scale == 64 ** -0.5
    q2, _, _, _ = attention.input_helper(1, 4, 2, 64, 96, 64, torch.float32, "bshd", device="cpu")
    assert torch.equal(q, q2)


def test_launcher_rejects_cpu_tensors_and_causal():
    q = torch.zeros(1, 2, 128, 64, dtype=torch.float16)
    md = attention.MetaData(0.1)
    md.layout = "bhsd"
    with pytest.raises(ValueError, match="CUDA"):
        attention.run_gluon_attention(q, q, q, torch.empty_like(q), md)
    md.causal = True
    with pytest.raises(AssertionError):
        attention.run_gluon_attention(q, q, q, torch.empty_like(q), md)


# ------------------------------------------------------ C-ABI arguments --
def _call(strides=None, B=1, HQ=2, HK=2, Sq=128, Sk=128, D=128, dtype=None, scale=0.1,
          ptrs=(4096, 8192, 12288, 16384)):
    if strides is None:
        strides = [HQ * Sq * D, Sq * D, D, 1] * 4
    arr = (ctypes.c_int64 * 16)(*strides)
    return _lib.lib().b2g_attention_fwd(*ptrs, arr, B, HQ, HK, Sq, Sk, D,
                                        _lib.DT_BF16 if dtype is None else dtype, scale,
                                        None, None, None)


@pytest.mark.parametrize("kw,code", [
    (dict(D=96), _lib.ESHAPE),
    (dict(D=256), _lib.ESHAPE),
    (dict(HQ=3, HK=2), _lib.ESHAPE),
    (dict(Sk=0), _lib.ESHAPE),
    (dict(Sq=-1), _lib.ESHAPE),
    (dict(B=0), _lib.ESHAPE),
    (dict(dtype=_lib.DT_F32), _lib.EINVAL),
    (dict(scale=0.0), _lib.EINVAL),
    (dict(scale=float("nan")), _lib.EINVAL),
    (dict(ptrs=(0, 8192, 12288, 16384)), _lib.EINVAL),
    (dict(ptrs=(4097, 8192, 12288, 16384)), _lib.EALIGN),
    (dict(strides=[256 * 128, 128 * 128, 128, 2] + [256 * 128, 128 * 128, 128, 1] * 3),
     _lib.ESTRIDE),
    (dict(strides=[256 * 128, 128 * 128, 100, 1] + [256 * 128, 128 * 128, 128, 1] * 3),
     _lib.ESTRIDE),
    (dict(strides=[256 * 128, 128 * 128, 132, 1] + [256 * 128, 128 * 128, 128, 1] * 3),
     _lib.EALIGN),
], ids=lambda x: str(x) if not isinstance(x, dict) else ",".join(sorted(x)))
def test_attention_argument_errors(kw, code):
    assert _call(**kw) == code


def test_attention_lse_must_be_float_aligned():
    arr = (ctypes.c_int64 * 16)(*([2 * 128 * 128, 128 * 128, 128, 1] * 4))
    rc = _lib.lib().b2g_attention_fwd(4096, 8192, 12288, 16384, arr, 1, 2, 2, 128, 128, 128,
                                      _lib.DT_BF16, 0.1, 4098, None, None)
    assert rc == _lib.EALIGN


def test_attention_strides_pointer_required():
    rc = _lib.lib().b2g_attention_fwd(4096, 8192, 12288, 16384, None, 1, 2, 2, 128, 128, 128,
                                      _lib.DT_BF16, 0.1, None, None, None)
    assert rc == _lib.EINVAL


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device answer")
def test_attention_without_device_reports_it():
    assert _call() == _lib.ENODEVICE
