"""The C-ABI library loads, exports exactly what include/b2g.h declares, and
rejects bad arguments before touching a GPU (no compute calls here)."""

from __future__ import annotations

import ctypes
import os
import re
import subprocess

import pytest
from conftest import ROOT

from gfx950_gluon_tutorials_b200 import _lib

HEADER = os.path.join(ROOT, "include", "b2g.h")


def declared_functions() -> set[str]:
    text = open(HEADER).read()
    return set(re.findall(r"^B2G_API\s+[\w\s\*]+?\b(b2g_\w+)\(", text, flags=re.M))


def test_header_and_binding_agree():
    assert declared_functions() == set(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    for name in declared_functions():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\b(b2g_\w+)\b", out))
    assert exported == declared_functions()


def test_constants_match_header():
    text = open(HEADER).read()
    consts = dict(re.findall(r"#define (B2G_\w+) (-?0x[0-9a-fA-F]+|-?\d+)", text))
    for name, value in consts.items():
        py = name[len("B2G_"):]
        if hasattr(_lib, py):
            assert getattr(_lib, py) == int(value, 0), name


def test_version_and_strerror():
    lib = _lib.lib()
    assert lib.b2g_version() >= 100
    for code in (0, -1, -2, -3, -4, -5, -6, -7, -8, 0x1006):
        assert _lib.strerror(code)


def _f16(**kw):
    args = dict(A=16, lda=64, B=16, ldb=64, C=16, ldc=64, M=64, N=64, K=64, ind=0, outd=0,
                ws=None, wsb=0, st=None, stream=None)
    args.update(kw)
    return _lib.lib().b2g_gemm_f16(*args.values())


@pytest.mark.parametrize("kw,code", [
    (dict(A=None), _lib.EINVAL),
    (dict(ind=7), _lib.EINVAL),
    (dict(outd=2), _lib.EINVAL),
    (dict(M=0), _lib.ESHAPE),
    (dict(K=-3), _lib.ESHAPE),
    (dict(A=24), _lib.EALIGN),          # not 16-byte aligned
    (dict(lda=60), _lib.EALIGN),        # 120-byte rows
    (dict(lda=68), _lib.EALIGN),        # 136-byte rows
    (dict(lda=32), _lib.ESTRIDE),       # row stride shorter than K
    (dict(ldc=32), _lib.ESTRIDE),
])
def test_gemm_f16_argument_errors(kw, code):
    assert _f16(**kw) == code


def test_gemm_scaled_argument_errors():
    lib = _lib.lib()
    # one scale pointer without the other
    rc = lib.b2g_gemm_f8(16, 64, 16, 64, 16, 1, 64, None, 0, 0, 16, 64, 64, 64, 64, 1,
                         None, 0, None, None)
    assert rc == _lib.EINVAL
    # scaled e5m2 needs K % 32 == 0
    rc = lib.b2g_gemm_f8(16, 64, 16, 64, 16, 1, 64, 16, 1, 64, 16, 64, 64, 64, 48, 1,
                         None, 0, None, None)
    assert rc == _lib.ESHAPE
    # mxfp4 without scales
    rc = lib.b2g_gemm_mxf4(16, 32, 16, 32, None, 0, 0, None, 0, 0, 16, 64, 64, 64, 64, 1,
                           None, 0, None, None)
    assert rc == _lib.EINVAL


def test_quant_argument_errors():
    lib = _lib.lib()
    assert lib.b2g_quant_mxfp4(16, 64, 4, 48, 16, 32, 16, 1, 4, None) == _lib.ESHAPE
    assert lib.b2g_quant_mxfp4(20, 64, 4, 64, 16, 32, 16, 1, 4, None) == _lib.EALIGN
    assert lib.b2g_quant_mxe5m2(16, 64, 4, 64, None, 1, 4, 16, 64, None) == _lib.EINVAL
    assert lib.b2g_cast_e5m2(16, 9, 10, 16, None) == _lib.EINVAL
    assert lib.b2g_cast_e5m2(16, 2, 0, 16, None) == _lib.OK  # empty: nothing to launch


def test_options_roundtrip():
    old = _lib.get_option(_lib.OPT_SK_MODE)
    try:
        _lib.set_option(_lib.OPT_SK_MODE, 2)
        assert _lib.get_option(_lib.OPT_SK_MODE) == 2
        with pytest.raises(_lib.B2GError):
            _lib.set_option(_lib.OPT_SK_MODE, 9)
    finally:
        _lib.set_option(_lib.OPT_SK_MODE, old)
    assert _lib.lib().b2g_set_option(999, 1) == _lib.EINVAL
    assert _lib.get_option(_lib.OPT_SKINNY_MAX_M) == 128
    assert _lib.lib().b2g_set_option(_lib.OPT_SKINNY_MAX_M, 129) == _lib.EINVAL


def test_prepare_gemm_argument_errors():
    """Preparation checks the same arguments as the direct entry points before
    touching a device, leaves the handle null on failure, and the run and free
    entry points accept a null handle."""
    lib = _lib.lib()
    out = ctypes.c_void_p(12345)

    def prep(kind=_lib.KIND_F16, A=16, sfa=None, sfb=None, K=64, outp=ctypes.byref(out)):
        return lib.b2g_prepare_gemm(kind, A, 64, 16, 64, sfa, 1, 64, sfb, 1, 64, 16, 64, 64, 64,
                                    K, 0, None, 0, None, outp)

    assert prep(outp=None) == _lib.EINVAL
    assert prep(kind=9) == _lib.EINVAL and out.value is None
    assert prep(sfa=16, sfb=16) == _lib.EINVAL          # scales on an unscaled kind
    assert prep(kind=_lib.KIND_MXFP4) == _lib.EINVAL     # scaled kind without scales
    assert prep(A=24) == _lib.EALIGN
    assert prep(kind=_lib.KIND_MXE5M2, sfa=16, sfb=16, K=48) == _lib.ESHAPE
    assert out.value is None
    assert lib.b2g_prepared_run(None, None) == _lib.EINVAL
    lib.b2g_prepared_free(None)
