"""Drop-in for the reference's a4w4 (MXFP4) ``matmul_kernel`` modules.

``matmul(a, b, a_scales, b_scales)`` mirrors
kernels/gemm/intra_wave/a4w4/v1_sliceMN/matmul_kernel.py:696-742: A (M, K/2) and
B (N, K/2) packed e2m1 bytes (even k in the low nibble), E8M0 scales
(M, K/32) and (N, K/32) with any strides (the reference's own are
M-contiguous), bf16 output. ``matmul_kernel_only`` takes a preallocated C like
kernels/gemm/inter_wave/a4w4/v2_mfma32x32x64/matmul_kernel.py:614-668.
"""

from __future__ import annotations

import torch

from . import ops
from .ops import gemm_mxf4

BLOCK_M, BLOCK_N, BLOCK_K = 128, 256, 256
MIN_K = 32
KERNEL_NAME = "gemm_kernel"


def matmul(a: torch.Tensor, b: torch.Tensor, a_scales: torch.Tensor,
           b_scales: torch.Tensor, c: torch.Tensor | None = None) -> torch.Tensor:
    return gemm_mxf4(a, b, a_scales, b_scales, c)


def matmul_kernel_only(a: torch.Tensor, b: torch.Tensor, a_scales: torch.Tensor,
                       b_scales: torch.Tensor, c: torch.Tensor) -> torch.Tensor:
    return gemm_mxf4(a, b, a_scales, b_scales, c)


def grouped_matmul(a: torch.Tensor, b_experts: torch.Tensor, a_scales: torch.Tensor,
                   b_scales, group_offsets: torch.Tensor,
                   c: torch.Tensor | None = None) -> torch.Tensor:
    """MoE grouped MXFP4 GEMM (the reference's roadmap item "4-bit MoE kernel",
    ROADMAP.md): rows [g[e], g[e+1]) of `a` are multiplied by expert e's
    weights b_experts[e]; see ops.gemm_mxf4_grouped for the layout rules."""
    return ops.gemm_mxf4_grouped(a, b_experts, a_scales, b_scales, group_offsets, c=c)
