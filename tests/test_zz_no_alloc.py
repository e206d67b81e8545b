"""b2g_gemm_mxf4_noalloc: the a4w4 GEMM on the library's static per-device
scratch, called through the C ABI and checked against b2g_gemm_mxf4 (the
workspace entry point) on the same inputs, two calls in a row.

This file is collected last so that it also runs after every other test has
set options, loaded kernels and left workspaces behind; it passes alone too.
"""

from __future__ import annotations

import json
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from gfx950_gluon_tutorials_b200 import _lib, ops
from oracle import mx

pytestmark = pytest.mark.gpu

TOL_F4 = 3e-2   # normalised max-abs error bound for MXFP4 outputs


def _noalloc(a, b, sa, sb, c, status) -> int:
    """One b2g_gemm_mxf4_noalloc call; the scales keep their (any-order) strides."""
    M, Kp = a.shape
    N = b.shape[0]
    return _lib.lib().b2g_gemm_mxf4_noalloc(
        a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0),
        sa.data_ptr(), sa.stride(0), sa.stride(1), sb.data_ptr(), sb.stride(0), sb.stride(1),
        c.data_ptr(), c.stride(0), M, N, 2 * Kp, _lib.DT_BF16,
        status.data_ptr(), torch.cuda.current_stream().cuda_stream)


def _quantised(M, N, K, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    qa, sa = ops.quantize_mxfp4(torch.randn((M, K), generator=gen, device="cuda"))
    qb, sb = ops.quantize_mxfp4(torch.randn((N, K), generator=gen, device="cuda"))
    return qa, qb, sa, sb


@pytest.mark.parametrize("shape", [(4096, 4096, 8192), (1000, 600, 2048), (128, 256, 256)],
                         ids=lambda s: "x".join(map(str, s)))
def test_noalloc_matches_workspace_entry_point(cuda_device, shape):
    M, N, K = shape
    need = _lib.lib().b2g_gemm_workspace_bytes(_lib.KIND_MXFP4, M, N, K)
    assert 0 < need <= _lib.NOALLOC_SCRATCH_BYTES
    qa, qb, sa, sb = _quantised(M, N, K, seed=M + N + K)
    ref = ops.gemm_mxf4(qa, qb, sa, sb)
    ops.check_status()
    ref32 = ref.float().cpu().numpy()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    outs = [torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
            for _ in range(2)]
    torch.cuda.synchronize()
    for i, c in enumerate(outs):
        rc = _noalloc(qa, qb, sa, sb, c, status)
        assert rc == _lib.OK, _lib.lib().b2g_strerror(rc).decode()
        torch.cuda.synchronize()
        assert int(status.item()) == 0, _lib.lib().b2g_strerror(int(status.item())).decode()
        err = mx.normalised_max_abs(c.float().cpu().numpy(), ref32)
        assert err <= TOL_F4, f"call {i}: normalised max-abs error {err:.3e} > {TOL_F4}"


def test_noalloc_matches_oracle_on_reference_recipe(cuda_device):
    """Reference input recipe (random nibbles, E8M0 bytes 124..127, M-contiguous
    A scales) against the CPU restatement, for both of two consecutive calls."""
    M, N, K = 200, 320, 1024
    g = torch.Generator().manual_seed(7)
    a = torch.randint(0, 256, (M, K // 2), generator=g, dtype=torch.uint8)
    b = torch.randint(0, 256, (N, K // 2), generator=g, dtype=torch.uint8)
    sa = torch.randint(124, 128, (K // 32, 256), generator=g, dtype=torch.uint8).T[:M]
    sb = torch.randint(124, 128, (K // 32, N), generator=g, dtype=torch.uint8).T
    ref = mx.bf16_bits_to_f32(mx.gemm_mxfp4_ref(a.numpy(), b.numpy(), sa.numpy(), sb.numpy()))
    a, b, sa, sb = a.cuda(), b.cuda(), sa.cuda(), sb.cuda()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    for i in range(2):
        c = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
        rc = _noalloc(a, b, sa, sb, c, status)
        assert rc == _lib.OK, _lib.lib().b2g_strerror(rc).decode()
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        err = mx.normalised_max_abs(c.float().cpu().numpy(), ref)
        assert err <= TOL_F4, f"call {i}: normalised max-abs error {err:.3e} > {TOL_F4}"


def test_noalloc_rejects_problems_beyond_its_capacity(cuda_device):
    """Deep K makes the relaid scales alone 32 MiB: refused before any launch,
    and the entry point still works afterwards."""
    M, N, K = 4096, 4096, 131072
    need = _lib.lib().b2g_gemm_workspace_bytes(_lib.KIND_MXFP4, M, N, K)
    assert need > _lib.NOALLOC_SCRATCH_BYTES
    a = torch.zeros((M, K // 2), dtype=torch.uint8, device="cuda")
    b = torch.zeros((N, K // 2), dtype=torch.uint8, device="cuda")
    sa = torch.full((M, K // 32), 127, dtype=torch.uint8, device="cuda")
    sb = torch.full((N, K // 32), 127, dtype=torch.uint8, device="cuda")
    c = torch.full((M, N), 3.0, dtype=torch.bfloat16, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = _noalloc(a, b, sa, sb, c, status)
    assert rc == _lib.ECAPACITY
    assert "capacity" in _lib.lib().b2g_strerror(rc).decode()
    torch.cuda.synchronize()
    assert bool((c == 3.0).all()), "a rejected call must not write C"
    del a, b, sa, sb, c
    qa, qb, sa, sb = _quantised(256, 512, 1024, seed=5)
    ref = ops.gemm_mxf4(qa, qb, sa, sb).float().cpu().numpy()
    c = torch.empty((256, 512), dtype=torch.bfloat16, device="cuda")
    assert _noalloc(qa, qb, sa, sb, c, status) == _lib.OK
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert mx.normalised_max_abs(c.float().cpu().numpy(), ref) <= TOL_F4


def test_noalloc_argument_errors_match_workspace_entry_point(cuda_device):
    """Argument checks run before the capacity check and give the same codes."""
    a = torch.zeros((128, 128), dtype=torch.uint8, device="cuda")
    s = torch.full((128, 8), 127, dtype=torch.uint8, device="cuda")
    c = torch.empty((128, 128), dtype=torch.bfloat16, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    lib = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    st = status.data_ptr()
    # K not a multiple of 32
    rc = lib.b2g_gemm_mxf4_noalloc(a.data_ptr(), 128, a.data_ptr(), 128, s.data_ptr(), 8, 1,
                                   s.data_ptr(), 8, 1, c.data_ptr(), 128, 128, 128, 250,
                                   _lib.DT_BF16, st, stream)
    assert rc == _lib.ESHAPE
    # missing scales
    rc = lib.b2g_gemm_mxf4_noalloc(a.data_ptr(), 128, a.data_ptr(), 128, None, 0, 0, None, 0,
                                   0, c.data_ptr(), 128, 128, 128, 256, _lib.DT_BF16, st, stream)
    assert rc == _lib.EINVAL
    assert np.all(status.cpu().numpy() == 0)


# Run in a fresh interpreter: CUPTI's driver-API callbacks count every device
# or pinned-host allocation and free the process makes while the second
# no-allocation call runs, including an allocation freed again before the
# call returns (which a device-wide free-memory reading cannot see).
_COUNT_SCRIPT = r"""
import ctypes, json, os, sys
sys.path.insert(0, sys.argv[1])
import torch
from gfx950_gluon_tutorials_b200 import _lib, ops
from oracle import mx

# cupti_driver_cbid.h: cuMemAlloc{,_v2}, cuMemAllocPitch{,_v2}, cuMemAllocHost{,_v2},
# cuMemHostAlloc{,_v2}, cuMemAllocManaged, cuMemCreate, cuMemAllocAsync{,_ptsz},
# cuMemAllocFromPoolAsync{,_ptsz}, cuMemFree{,_v2}, cuMemFreeHost, cuMemRelease,
# cuMemFreeAsync{,_ptsz}, cuMemPoolCreate
CBIDS = [29, 243, 31, 244, 37, 294, 39, 271, 371, 549, 598, 599, 611, 612,
         33, 245, 38, 550, 600, 601, 607]
calls = []
ok = False
try:
    import nvidia.cuda_cupti as cp
    cupti = ctypes.CDLL(os.path.join(os.path.dirname(cp.__file__), "lib", "libcupti.so.12"))
    CB = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_int, ctypes.c_uint32, ctypes.c_void_p)
    def on_call(user, domain, cbid, data):
        if ctypes.cast(data, ctypes.POINTER(ctypes.c_int))[0] == 0:   # API enter
            calls.append(int(cbid))
    cb = CB(on_call)
    sub = ctypes.c_void_p()
    ok = cupti.cuptiSubscribe(ctypes.byref(sub), cb, None) == 0
    if ok:
        ok = all(cupti.cuptiEnableCallback(1, sub, 1, c) == 0 for c in CBIDS)
except Exception as e:  # noqa: BLE001
    ok = False
torch.cuda.set_device(0)
M, N, K = 1024, 768, 2048
gen = torch.Generator(device="cuda").manual_seed(21)
qa, sa = ops.quantize_mxfp4(torch.randn((M, K), generator=gen, device="cuda"))
qb, sb = ops.quantize_mxfp4(torch.randn((N, K), generator=gen, device="cuda"))
ref = ops.gemm_mxf4(qa, qb, sa, sb).float().cpu().numpy()
status = torch.zeros(1, dtype=torch.int32, device="cuda")
outs = [torch.empty((M, N), dtype=torch.bfloat16, device="cuda") for _ in range(2)]
stream = torch.cuda.current_stream().cuda_stream
def call(c):
    return _lib.lib().b2g_gemm_mxf4_noalloc(
        qa.data_ptr(), qa.stride(0), qb.data_ptr(), qb.stride(0), sa.data_ptr(), sa.stride(0),
        sa.stride(1), sb.data_ptr(), sb.stride(0), sb.stride(1), c.data_ptr(), c.stride(0),
        M, N, K, _lib.DT_BF16, status.data_ptr(), stream)
rc0 = call(outs[0])                      # first call on this device: set-up
torch.cuda.synchronize()
free0 = torch.cuda.mem_get_info()[0]
del calls[:]
rc1 = call(outs[1])
torch.cuda.synchronize()
seen = list(calls)
free1 = torch.cuda.mem_get_info()[0]
errs = [mx.normalised_max_abs(o.float().cpu().numpy(), ref) for o in outs]
print(json.dumps({"cupti": ok, "rc": [rc0, rc1], "status": int(status.item()),
                  "alloc_calls": seen, "free_drop": free0 - free1, "errs": errs}))
"""


def test_noalloc_second_call_makes_no_allocation_calls(cuda_device):
    """The call after set-up makes no device or pinned-host allocation or free
    (counted with CUPTI driver-API callbacks in a fresh process) and matches
    the workspace entry point. Without CUPTI, the device's free memory must
    not drop by an allocation's 2 MiB granule across the call."""
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", _COUNT_SCRIPT, root], capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    res = json.loads(r.stdout.strip().splitlines()[-1])
    assert res["rc"] == [_lib.OK, _lib.OK], res
    assert res["status"] == 0, res
    assert max(res["errs"]) <= TOL_F4, res
    if res["cupti"]:
        assert res["alloc_calls"] == [], f"allocation calls during the call: {res['alloc_calls']}"
    else:
        assert res["free_drop"] < (2 << 20), f"free device memory dropped by {res['free_drop']}"
