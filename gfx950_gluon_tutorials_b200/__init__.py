"""B200-native (sm_100a) GEMM hot path of gfx950-gluon-tutorials.

C = A @ B^T in FP16/BF16 (``a16w16``), BF8 = E5M2 (``a8w8``) and MXFP4
(``a4w4``) through the C ABI of ``libb2g.so`` (include/b2g.h), plus the
quantise-and-pack kernels (``ops.quantize_mxfp4``, ``ops.quantize_mxe5m2``,
``ops.cast_e5m2``). The submodules ``a16w16``, ``a8w8`` and ``a4w4`` keep the
reference's ``matmul`` signatures so its bench drivers can import them.
``attention`` is the flash-attention forward behind the reference's
``run_gluon_attention`` launcher.
"""

from . import a4w4, a8w8, a16w16, attention, ops  # noqa: F401
from ._lib import B2GError, LIB_PATH, lib  # noqa: F401

__all__ = ["a16w16", "a8w8", "a4w4", "attention", "ops", "B2GError", "lib", "LIB_PATH"]
