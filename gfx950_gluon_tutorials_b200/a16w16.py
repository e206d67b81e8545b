"""Drop-in for the reference's a16w16 ``matmul_kernel`` modules.

Mirrors ``matmul(a, b, c=None)`` of
kernels/gemm/intra_wave/a16w16/v9_beyond_hotloop/matmul_kernel.py:390-424 and
``matmul_kernel_only(a, b_t, c)`` / ``matmul(a, b, c=None)`` of
kernels/gemm/inter_wave/a16w16/matmul_kernel.py:335-379: same argument meaning,
same assertions, C allocated in ``a.dtype`` when not given, asynchronous on the
current stream. The work runs in the sm_100a ``kind::f16`` kernel of libb2g.so.
"""

from __future__ import annotations

import torch

from .ops import gemm_f16

# Output tile of one CTA pair (cta_group::2) and K per pipeline stage.
BLOCK_M, BLOCK_N, BLOCK_K = 256, 256, 64
MIN_K = 1
KERNEL_NAME = "gemm_kernel"


def matmul_kernel_only(a: torch.Tensor, b_t: torch.Tensor, c: torch.Tensor) -> torch.Tensor:
    """C = A @ B_t^T with ``b_t`` already (N, K) K-contiguous and ``c`` preallocated."""
    return gemm_f16(a, b_t, c)


def matmul(a: torch.Tensor, b: torch.Tensor, c: torch.Tensor | None = None) -> torch.Tensor:
    """C = A @ B with ``b`` a (K, N) tensor, usually the transposed view of an
    (N, K) K-contiguous buffer as the reference's bench builds it."""
    assert a.shape[1] == b.shape[0], "Incompatible dimensions"
    assert a.is_contiguous(), "Matrix A must be contiguous"
    b_t = b.T
    if b_t.stride(1) != 1:
        b_t = b_t.contiguous()
    if c is None:
        c = torch.empty((a.shape[0], b.shape[1]), device=a.device, dtype=a.dtype)
    return gemm_f16(a, b_t, c)
