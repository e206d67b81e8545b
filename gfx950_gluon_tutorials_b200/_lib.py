"""ctypes binding of libb2g.so (the C ABI declared in include/b2g.h).

The library is built in-tree by ``python -m gfx950_gluon_tutorials_b200.build``
(``__graft_entry__.build()`` does the same). There is no fallback: if the
shared object is missing, every entry point raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libb2g.so")

# Constants mirrored from include/b2g.h
KIND_F16, KIND_BF16, KIND_E5M2, KIND_MXE5M2, KIND_MXFP4 = 0, 1, 2, 3, 4
DT_F16, DT_BF16, DT_F32 = 0, 1, 2
OK = 0
EINVAL, ESHAPE, EALIGN, ESTRIDE, EWORKSPACE, ETENSORMAP, ENODEVICE, ECAPACITY = (
    -1, -2, -3, -4, -5, -6, -7, -8)
STATUS_TIMEOUT = 0x1000
STATUS_SMEM_BASE = 0x2000
STATUS_BAD_GROUPS = 0x3000
SITE_EMPTY, SITE_FULL, SITE_ACC_EMPTY, SITE_ACC_FULL, SITE_OVERLAP, SITE_FLAG = 1, 2, 3, 4, 5, 6
SITE_SCALES = 7
OPT_PAIR, OPT_SK_MODE, OPT_GROUP_M, OPT_MIN_SK_ITERS, OPT_TIMEOUT_MS = 1, 2, 3, 4, 5
OPT_INJECT_FLAG_TIMEOUT, OPT_MAX_UNITS, OPT_L2_PREFETCH, OPT_SKINNY_MAX_M = 6, 7, 8, 9
OPT_SKINNY_SPLITS, OPT_SERPENTINE = 10, 11
NOALLOC_SCRATCH_BYTES = 32 << 20

_c_int, _c_i64, _c_sz, _vp = ctypes.c_int, ctypes.c_int64, ctypes.c_size_t, ctypes.c_void_p
_i32p = ctypes.POINTER(ctypes.c_int32)

# name -> (restype, argtypes); every function declared in include/b2g.h
SIGNATURES = {
    "b2g_version": (_c_int, []),
    "b2g_strerror": (ctypes.c_char_p, [_c_int]),
    "b2g_gemm_workspace_bytes": (_c_sz, [_c_int, _c_int, _c_int, _c_int]),
    "b2g_workspace_reset": (_c_int, [_vp, _c_sz, _vp]),
    "b2g_gemm_f16": (_c_int, [_vp, _c_i64, _vp, _c_i64, _vp, _c_i64, _c_int, _c_int, _c_int,
                              _c_int, _c_int, _vp, _c_sz, _vp, _vp]),
    "b2g_gemm_f8": (_c_int, [_vp, _c_i64, _vp, _c_i64, _vp, _c_i64, _c_i64, _vp, _c_i64, _c_i64,
                             _vp, _c_i64, _c_int, _c_int, _c_int, _c_int, _vp, _c_sz, _vp, _vp]),
    "b2g_gemm_mxf4": (_c_int, [_vp, _c_i64, _vp, _c_i64, _vp, _c_i64, _c_i64, _vp, _c_i64,
                               _c_i64, _vp, _c_i64, _c_int, _c_int, _c_int, _c_int, _vp, _c_sz,
                               _vp, _vp]),
    "b2g_gemm_mxf4_grouped": (_c_int, [_vp, _c_i64, _vp, _c_i64, _vp, _c_i64, _c_i64, _vp,
                                       _c_i64, _c_i64, _vp, _c_i64, _vp, _c_int, _c_int, _c_int,
                                       _c_int, _c_int, _vp, _c_sz, _vp, _vp]),
    "b2g_gemm_grouped_workspace_bytes": (_c_sz, [_c_int, _c_int, _c_int, _c_int]),
    "b2g_prepare_gemm": (_c_int, [_c_int, _vp, _c_i64, _vp, _c_i64, _vp, _c_i64, _c_i64, _vp,
                                  _c_i64, _c_i64, _vp, _c_i64, _c_int, _c_int, _c_int, _c_int,
                                  _vp, _c_sz, _vp, ctypes.POINTER(_vp)]),
    "b2g_prepared_run": (_c_int, [_vp, _vp]),
    "b2g_prepared_free": (None, [_vp]),
    "b2g_attention_fwd": (_c_int, [_vp, _vp, _vp, _vp, ctypes.POINTER(ctypes.c_int64), _c_int,
                                   _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
                                   ctypes.c_float, _vp, _vp, _vp]),
    "b2g_selftest_poly_exp2": (_c_int, [_vp, _vp, _vp, _vp, _c_i64, _vp]),
    "b2g_gemm_mxf4_noalloc": (_c_int, [_vp, _c_i64, _vp, _c_i64, _vp, _c_i64, _c_i64, _vp,
                                       _c_i64, _c_i64, _vp, _c_i64, _c_int, _c_int, _c_int,
                                       _c_int, _vp, _vp]),
    "b2g_quant_mxfp4": (_c_int, [_vp, _c_i64, _c_int, _c_int, _vp, _c_i64, _vp, _c_i64, _c_i64,
                                 _vp]),
    "b2g_quant_mxe5m2": (_c_int, [_vp, _c_i64, _c_int, _c_int, _vp, _c_i64, _c_i64, _vp, _c_i64,
                                  _vp]),
    "b2g_cast_e5m2": (_c_int, [_vp, _c_int, _c_i64, _vp, _vp]),
    "b2g_scales_blocked_bytes": (_c_sz, [_c_int, _c_int]),
    "b2g_scales_to_blocked": (_c_int, [_vp, _c_i64, _c_i64, _c_int, _c_int, _vp, _vp]),
    "b2g_set_option": (_c_int, [_c_int, _c_i64]),
    "b2g_get_option": (_c_i64, [_c_int]),
    "b2g_plan_query": (_c_int, [_c_int, _c_int, _c_int, _c_int, _c_int, _i32p, _c_int]),
    "b2g_plan_items": (_c_int, [_c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _i32p, _c_int]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class B2GError(RuntimeError):
    """A C-ABI call returned a nonzero code, or a kernel reported a status."""

    def __init__(self, code: int, what: str = ""):
        self.code = code
        msg = strerror(code) if _lib is not None else str(code)
        super().__init__(f"{what + ': ' if what else ''}{msg} (code {code})")


def lib() -> ctypes.CDLL:
    """Loads libb2g.so once; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with "
                    "`python -m gfx950_gluon_tutorials_b200.build` (there is no CPU fallback)")
            handle = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def strerror(code: int) -> str:
    return lib().b2g_strerror(int(code)).decode()


def check(code: int, what: str = "") -> None:
    if code != OK:
        raise B2GError(int(code), what)


def set_option(key: int, value: int) -> None:
    check(lib().b2g_set_option(key, int(value)), "b2g_set_option")


def get_option(key: int) -> int:
    return int(lib().b2g_get_option(key))
