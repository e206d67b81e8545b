"""Drop-in for the reference's a4w4 (MXFP4) ``matmul_kernel`` modules.

Shape contract (kernels/gemm/intra_wave/a4w4/v1_sliceMN/matmul_kernel.py:696-705,
kernels/gemm/inter_wave/a4w4/v2_mfma32x32x64/matmul_kernel.py:614-668):
A is (M, K//2) and B is (N, K//2) packed e2m1 bytes, K-contiguous, even k in
the low nibble; M = a.shape[0], K = 2 * a.shape[1], N = b.shape[0]; E8M0
scales are (M, K//32) and (N, K//32) with any strides (the reference's own are
M-contiguous); C is (M, N) bf16. ``matmul`` allocates C when it is not given
(the intra v1 wrapper always allocates, the inter v2 one takes ``c=None``);
``matmul_kernel_only`` writes into a preallocated C.
"""

from __future__ import annotations

import torch

from . import ops

BLOCK_M, BLOCK_N, BLOCK_K = 128, 256, 256
MIN_K = 32
KERNEL_NAME = "gemm_kernel"


def matmul_kernel_only(a: torch.Tensor, b: torch.Tensor, a_scales: torch.Tensor,
                       b_scales: torch.Tensor, c: torch.Tensor) -> torch.Tensor:
    """C = dequant(A) @ dequant(B).T into the preallocated bf16 C (M, N)."""
    if c is None:
        raise ValueError("matmul_kernel_only writes into a preallocated C")
    M, N = a.shape[0], b.shape[0]
    if a.shape[1] != b.shape[1]:
        raise ValueError("Incompatible dimensions")
    if tuple(c.shape) != (M, N) or c.dtype != torch.bfloat16:
        raise ValueError(f"c must be ({M}, {N}) bf16, got {tuple(c.shape)} {c.dtype}")
    return ops.gemm_mxf4(a, b, a_scales, b_scales, c)


def matmul(a: torch.Tensor, b: torch.Tensor, a_scales: torch.Tensor,
           b_scales: torch.Tensor, c: torch.Tensor | None = None) -> torch.Tensor:
    """C = dequant(A) @ dequant(B).T; a fresh bf16 (M, N) C unless `c` is given."""
    if c is None:
        c = torch.empty((a.shape[0], b.shape[0]), device=a.device, dtype=torch.bfloat16)
    return matmul_kernel_only(a, b, a_scales, b_scales, c)


def grouped_matmul(a: torch.Tensor, b_experts: torch.Tensor, a_scales: torch.Tensor,
                   b_scales, group_offsets: torch.Tensor,
                   c: torch.Tensor | None = None) -> torch.Tensor:
    """MoE grouped MXFP4 GEMM (the reference's roadmap item "4-bit MoE kernel",
    ROADMAP.md): rows [g[e], g[e+1]) of `a` are multiplied by expert e's
    weights b_experts[e]; see ops.gemm_mxf4_grouped for the layout rules."""
    return ops.gemm_mxf4_grouped(a, b_experts, a_scales, b_scales, group_offsets, c=c)
