"""Drop-in for the reference's a8w8 (BF8 = E5M2) ``matmul_kernel`` modules.

``matmul(a, b)`` mirrors kernels/gemm/intra_wave/a8w8/matmul_kernel.py:437-470
(unscaled e5m2 x e5m2, fp16 output, ``b`` a (K, N) view) and
``matmul_kernel_only`` mirrors kernels/gemm/inter_wave/a8w8/matmul_kernel.py:343-388.
``matmul_scaled`` adds the block-scaled form (E8M0 per 32 K, bf16 output) that
the B200 benchmark configuration asks for; it has no counterpart function in
the reference, whose a8w8 path is unscaled.
"""

from __future__ import annotations

import torch

from .ops import gemm_f8

BLOCK_M, BLOCK_N, BLOCK_K = 256, 256, 128
MIN_K = 1
KERNEL_NAME = "gemm_kernel"


def _bt(b: torch.Tensor) -> torch.Tensor:
    b_t = b.T
    return b_t if b_t.stride(1) == 1 else b_t.contiguous()


def matmul_kernel_only(a: torch.Tensor, b_t: torch.Tensor, c: torch.Tensor) -> torch.Tensor:
    return gemm_f8(a, b_t, c)


def matmul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    assert a.shape[1] == b.shape[0], "Incompatible dimensions"
    assert a.is_contiguous(), "Matrix A must be contiguous"
    c = torch.empty((a.shape[0], b.shape[1]), device=a.device, dtype=torch.float16)
    return gemm_f8(a, _bt(b), c)


def matmul_scaled(a: torch.Tensor, b: torch.Tensor, a_scales: torch.Tensor,
                  b_scales: torch.Tensor, c: torch.Tensor | None = None,
                  out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """C = (A * 2^(a_scales-127)) @ (B * 2^(b_scales-127)) with per-32-K E8M0 scales;
    ``b`` is (K, N) as in ``matmul``; a_scales (M, K/32), b_scales (N, K/32)."""
    assert a.shape[1] == b.shape[0], "Incompatible dimensions"
    return gemm_f8(a, _bt(b), c, a_scales=a_scales, b_scales=b_scales, out_dtype=out_dtype)
