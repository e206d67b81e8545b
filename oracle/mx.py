"""Numpy restatement of the reference's MX / FP8 encodings and GEMM checks.

Test infrastructure only (see oracle/__init__.py). Each function cites the
reference code it restates; the quantisers restate the rules the B200 build
defines (the reference draws random codes instead of quantising).
"""

from __future__ import annotations

import numpy as np

SCALE_GROUP_SIZE = 32  # kernels/gemm/intra_wave/a4w4/bench.py:77

# kernels/gemm/intra_wave/a4w4/bench.py:86-103: e2m1 code -> value
E2M1_VALUES = np.array(
    [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0],
    dtype=np.float32)


# ----------------------------------------------------------------- decoding --
def unpack_e2m1_codes(x: np.ndarray) -> np.ndarray:
    """(rows, K/2) packed bytes -> (rows, K) codes; the low nibble is element 2j
    (kernels/gemm/intra_wave/a4w4/bench.py:80-85)."""
    x = np.asarray(x, dtype=np.uint8)
    out = np.empty((x.shape[0], 2 * x.shape[1]), dtype=np.uint8)
    out[:, 0::2] = x & 0xF
    out[:, 1::2] = x >> 4
    return out


def mxfp4_to_f32(x: np.ndarray) -> np.ndarray:
    """kernels/gemm/intra_wave/a4w4/bench.py:80-105."""
    return E2M1_VALUES[unpack_e2m1_codes(x)]


def e8m0_to_f32(x: np.ndarray) -> np.ndarray:
    """2^(x-127), 255 -> NaN (kernels/gemm/intra_wave/a4w4/bench.py:108-112)."""
    x = np.asarray(x, dtype=np.uint8)
    with np.errstate(over="ignore"):  # 255 -> 2^128 overflows before it becomes NaN
        out = np.ldexp(np.float64(1.0), x.astype(np.int32) - 127).astype(np.float32)
    out[x == 255] = np.nan
    return out


def e5m2_to_f32(q: np.ndarray) -> np.ndarray:
    """e5m2 byte -> fp32 (e5m2 is the high byte of an fp16)."""
    q = np.asarray(q, dtype=np.uint8)
    return (q.astype(np.uint16) << 8).view(np.float16).astype(np.float32)


# ---------------------------------------------------------------- rounding --
def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bits, round to nearest even (torch's .to(bfloat16))."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_e5m2(y: np.ndarray) -> np.ndarray:
    """fp32 -> e5m2 bytes, round to nearest even, no saturation: |y| >= 61440
    (the tie above the largest finite value 57344) and inf -> inf, NaN -> 0x7F
    with the sign kept. This is the rounding of torch's float -> float8_e5m2
    cast (kernels/gemm/intra_wave/a8w8/bench.py:133-134 relies on it)."""
    y = np.ascontiguousarray(y, dtype=np.float32)
    u = y.view(np.uint32).astype(np.uint64)
    sign = ((u >> 24) & 0x80).astype(np.uint8)
    a = u & 0x7FFFFFFF
    out = np.zeros(y.shape, dtype=np.uint8)
    nan = a > 0x7F800000
    inf = (a >= 0x47700000) & ~nan
    normal = (a >= 0x38800000) & ~nan & ~inf
    sub = ~(nan | inf | normal)
    ar = a[normal] + 0xFFFFF + ((a[normal] >> 21) & 1)
    out[normal] = ((((ar >> 23) - 112) << 2) | ((ar >> 21) & 3)).astype(np.uint8)
    v = a[sub].astype(np.uint32).view(np.float32) * np.float32(65536.0)
    out[sub] = np.rint(v).astype(np.uint8)
    out[inf] = 0x7C
    out[nan] = 0x7F
    return out | sign


def e2m1_code(y: np.ndarray) -> np.ndarray:
    """fp32 -> e2m1 code: round to nearest even, saturate to +-6, sign kept
    (negative values that round to zero give the -0 code 8)."""
    y = np.ascontiguousarray(y, dtype=np.float32)
    a = np.abs(y)
    mag = np.full(y.shape, 7, dtype=np.uint8)
    # thresholds with ties to the even code (0.25->0, 0.75->1.0, 1.25->1.0,
    # 1.75->2, 2.5->2, 3.5->4, 5->4)
    for upper, inclusive, code in ((0.25, True, 0), (0.75, False, 1), (1.25, True, 2),
                                   (1.75, False, 3), (2.5, True, 4), (3.5, False, 5),
                                   (5.0, True, 6)):
        hit = (a <= upper) if inclusive else (a < upper)
        sel = hit & (mag == 7)
        mag[sel] = code
    sign = ((y.view(np.uint32) >> 28) & 0x8).astype(np.uint8)
    return mag | sign


def _floor_log2(a: np.ndarray) -> np.ndarray:
    """floor(log2(a)) for finite a > 0, exact (from the bits)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    e = (u >> 23).astype(np.int64)
    m = (u & 0x7FFFFF).astype(np.int64)
    sub = e == 0
    out = e - 127
    if np.any(sub):
        bl = np.array([int(v).bit_length() for v in m[sub]], dtype=np.int64)
        out[sub] = (bl - 1) - 149
    return out


def _exp2i(n: np.ndarray) -> np.ndarray:
    return np.ldexp(np.float64(1.0), n).astype(np.float32)


# --------------------------------------------------------------- quantisers --
def quantize_mxfp4(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """fp32 (rows, K) -> (packed (rows, K/2) uint8, scales (rows, K/32) uint8).

    Per 32-K block: s = floor(log2(max|x|)) - 2 clamped to >= -127 (E8M0 byte
    s + 127); all-zero block -> byte 0; a NaN/inf in the block -> byte 255 and
    zero codes; codes = e2m1(x * 2^-s); two codes per byte, even k low."""
    x = np.asarray(x, dtype=np.float32)
    rows, K = x.shape
    assert K % 32 == 0
    blk = x.reshape(rows, K // 32, 32)
    amax = np.max(np.abs(blk), axis=2)
    nonfinite = ~np.all(np.isfinite(blk), axis=2)
    zero = (amax == 0) & ~nonfinite
    ok = ~(nonfinite | zero)
    s = np.full(amax.shape, -127, dtype=np.int64)
    s[ok] = np.maximum(_floor_log2(amax[ok]) - 2, -127)
    scales = (s + 127).astype(np.uint8)
    scales[nonfinite] = 255
    scales[zero] = 0
    mul = _exp2i(-s)
    with np.errstate(over="ignore", invalid="ignore"):  # non-finite blocks are zeroed below
        y = blk * mul[:, :, None]
    codes = e2m1_code(y)
    codes[nonfinite] = 0
    codes = codes.reshape(rows, K)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
    return packed, scales


def quantize_mxe5m2(x: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """fp32 (rows, K), E8M0 (rows, K/32) -> e5m2 bytes of x * 2^-(e-127);
    a block with scale byte 255 gets zero codes."""
    x = np.asarray(x, dtype=np.float32)
    rows, K = x.shape
    e = np.asarray(scales, dtype=np.int64)
    mul = _exp2i(127 - e)
    with np.errstate(over="ignore", invalid="ignore"):  # overflow -> inf, as on the GPU
        y = x.reshape(rows, K // 32, 32) * mul[:, :, None]
    q = f32_to_e5m2(y)
    q[e == 255] = 0
    return q.reshape(rows, K)


# -------------------------------------------------------------- GEMM oracles --
def gemm_mxfp4_ref(a_fp4, b_fp4, a_scales, b_scales) -> np.ndarray:
    """torch_reference restated (kernels/gemm/intra_wave/a4w4/bench.py:149-164):
    dequantise both operands, fp32 A @ B^T, cast to bf16. Returns bf16 bits."""
    a = mxfp4_to_f32(a_fp4) * np.repeat(e8m0_to_f32(a_scales), SCALE_GROUP_SIZE, axis=1)
    b = mxfp4_to_f32(b_fp4) * np.repeat(e8m0_to_f32(b_scales), SCALE_GROUP_SIZE, axis=1)
    return f32_to_bf16_bits(a @ b.T)


def gemm_mxfp4_grouped_ref(a_fp4, b_fp4, a_scales, b_scales, offsets) -> np.ndarray:
    """Grouped a4w4 (MoE experts): gemm_mxfp4_ref per expert e on rows
    [offsets[e], offsets[e+1]) of A with rows [e*N, (e+1)*N) of B, where
    N = B rows / experts. No reference counterpart exists (its roadmap plans
    the kernel); the per-group product is the reference's torch_reference.
    Returns bf16 bits (M, N)."""
    offsets = np.asarray(offsets)
    E = len(offsets) - 1
    N = b_fp4.shape[0] // E
    out = np.zeros((a_fp4.shape[0], N), dtype=np.uint16)
    for e in range(E):
        r0, r1 = int(offsets[e]), int(offsets[e + 1])
        if r1 > r0:
            out[r0:r1] = gemm_mxfp4_ref(a_fp4[r0:r1], b_fp4[e * N:(e + 1) * N],
                                        a_scales[r0:r1], b_scales[e * N:(e + 1) * N])
    return out


def gemm_mxe5m2_ref(a_q, b_q, a_scales, b_scales) -> np.ndarray:
    """Scaled BF8 in the same dequantise-then-fp32-mm pattern; bf16 bits."""
    a = e5m2_to_f32(a_q) * np.repeat(e8m0_to_f32(a_scales), SCALE_GROUP_SIZE, axis=1)
    b = e5m2_to_f32(b_q) * np.repeat(e8m0_to_f32(b_scales), SCALE_GROUP_SIZE, axis=1)
    return f32_to_bf16_bits(a @ b.T)


def gemm_e5m2_ref(a_q, b_q) -> np.ndarray:
    """kernels/gemm/intra_wave/a8w8/bench.py:138: matmul of the fp16-upcast e5m2
    operands; fp32 accumulation, fp16 result."""
    return (e5m2_to_f32(a_q) @ e5m2_to_f32(b_q).T).astype(np.float16)


def gemm_f16_ref(a: np.ndarray, b_t: np.ndarray, out: str = "f16") -> np.ndarray:
    """kernels/gemm/intra_wave/a16w16/bench.py:183 (torch.matmul in the input
    dtype, fp32 accumulation). a, b_t are fp16 arrays or bf16 bit arrays
    (uint16); returns fp16 or bf16 bits."""
    def up(t):
        t = np.asarray(t)
        return bf16_bits_to_f32(t) if t.dtype == np.uint16 else t.astype(np.float32)
    c = up(a) @ up(b_t).T
    return c.astype(np.float16) if out == "f16" else f32_to_bf16_bits(c)


def normalised_max_abs(c, ref) -> float:
    """max|C - C_ref| / max|C_ref| (the tolerance metric the B200 build reports)."""
    c = np.asarray(c, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    denom = np.max(np.abs(ref))
    return float(np.max(np.abs(c - ref)) / (denom if denom > 0 else 1.0))
