"""CPU oracle for the attention forward pass - TEST INFRASTRUCTURE ONLY.

Restates the reference's correctness path for its FMHA forward kernel
(jamesbowley/gfx950-gluon-tutorials):
  - sdpa_ref: kernels/attention/common.py:115-138 (sdpa_reference): fp32
    softmax(Q K^T * sm_scale) V over a bhsd frame, K and V heads repeated
    (repeat_interleave) for grouped-query attention; non-causal only, as the
    tutorial kernel. Computed here in float64 so that it stands above both the
    reference's fp32 result and the kernel under test. It also returns the
    natural-log log-sum-exp of each row's scaled scores.
  - check_output: kernels/attention/common.py:142-174 (_check_output): the
    absolute floor grows to two ULPs of the output format at the largest
    reference magnitude, rtol 1e-3, elementwise |o - ref| <= atol + rtol*|ref|
    as torch.testing.assert_close applies it.

Pinned against tests/golden/attention_*.npz, produced by running the
reference's own sdpa_reference on the CPU (tests/golden/make_attention_golden.py).
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use it.
"""

from __future__ import annotations

import math

import numpy as np

# finfo(dtype).eps of the 16-bit output formats
EPS = {"float16": 2.0 ** -10, "bfloat16": 2.0 ** -7}


def sdpa_ref(q: np.ndarray, k: np.ndarray, v: np.ndarray, sm_scale: float | None = None
             ) -> tuple[np.ndarray, np.ndarray]:
    """O (B, HQ, Sq, D) and lse (B, HQ, Sq) for bhsd float arrays (common.py:115)."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(q.shape[-1])
    hq, hk = q.shape[1], k.shape[1]
    if hq != hk:
        r = hq // hk
        k = np.repeat(k, r, axis=1)
        v = np.repeat(v, r, axis=1)
    s = np.einsum("bhmd,bhnd->bhmn", q, k) * sm_scale
    mx = s.max(axis=-1, keepdims=True)
    e = np.exp(s - mx)
    den = e.sum(axis=-1, keepdims=True)
    o = np.einsum("bhmn,bhnd->bhmd", e / den, v)
    lse = (mx + np.log(den))[..., 0]
    return o, lse


def check_output(o: np.ndarray, o_ref: np.ndarray, out_dtype: str, atol: float = 1e-3,
                 rtol: float = 1e-3) -> tuple[bool, float, float]:
    """(ok, max |diff|, mean |diff|) under the reference's tolerance (common.py:142)."""
    o = np.asarray(o, dtype=np.float64)
    o_ref = np.asarray(o_ref, dtype=np.float64)
    scale = float(np.abs(o_ref).max()) if o_ref.size else 0.0
    if scale > 0 and math.isfinite(scale):
        atol = max(atol, 2 * EPS[out_dtype] * scale)
    diff = np.abs(o - o_ref)
    ok = bool(np.all(np.isfinite(o)) and np.all(diff <= atol + rtol * np.abs(o_ref)))
    return ok, float(diff.max()) if diff.size else 0.0, float(diff.mean()) if diff.size else 0.0


def sdpa_tiles(q: np.ndarray, k: np.ndarray, v: np.ndarray, sm_scale: float,
               rows: slice) -> np.ndarray:
    """O for a slice of query rows only, float64: lets a test check sampled rows
    of a problem too large to evaluate whole on the CPU."""
    return sdpa_ref(q[:, :, rows], k, v, sm_scale)[0]
