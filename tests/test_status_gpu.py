"""Failure detection without a GPU fault: a stream-K owner is made to wait for a
flag value no contributor ever writes. Its bounded wait expires after the
configured deadline, the kernel records the wait site in the device status
word and still finishes; the host raises, clears the workspace and the next
call on the same context is correct again."""

from __future__ import annotations

import pytest
import torch

from gfx950_gluon_tutorials_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def test_injected_flag_wait_times_out_and_context_recovers(cuda_device):
    keys = (_lib.OPT_INJECT_FLAG_TIMEOUT, _lib.OPT_TIMEOUT_MS, _lib.OPT_MIN_SK_ITERS,
            _lib.OPT_SK_MODE)
    old = {k: _lib.get_option(k) for k in keys}
    M, N, K = 512, 512, 4096   # 4 pair tiles on 74 pairs: every tile is split in k
    a = torch.randn((M, K), device="cuda", dtype=torch.float16)
    b_t = torch.randn((N, K), device="cuda", dtype=torch.float16)
    try:
        # split mode: the leftover tiles have owners that wait for contributors
        _lib.set_option(_lib.OPT_SK_MODE, 3)
        _lib.set_option(_lib.OPT_MIN_SK_ITERS, 1)
        p = ops.plan(_lib.KIND_F16, M, N, K,
                     torch.cuda.get_device_properties(0).multi_processor_count)
        assert p["splits"] > 1, p
        _lib.set_option(_lib.OPT_TIMEOUT_MS, 200)
        _lib.set_option(_lib.OPT_INJECT_FLAG_TIMEOUT, 1)
        ops.gemm_f16(a, b_t)
        with pytest.raises(ops.B2GError) as ei:
            ops.check_status(cuda_device)
        assert ei.value.code == _lib.STATUS_TIMEOUT | _lib.SITE_FLAG
    finally:
        for k, v in old.items():
            _lib.set_option(k, v)
    # same process, same context: a normal call works and is correct
    c = ops.gemm_f16(a, b_t)
    ops.check_status(cuda_device)
    ref = a.float() @ b_t.float().T
    err = ((c.float() - ref).abs().max() / ref.abs().max()).item()
    assert err < 1e-2
