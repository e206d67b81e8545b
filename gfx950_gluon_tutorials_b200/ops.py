"""Torch-facing calls into libb2g.so.

Every function launches asynchronously on the current torch CUDA stream and
returns without synchronising, as the reference's ``matmul`` wrappers do
(kernels/gemm/intra_wave/a16w16/v9_beyond_hotloop/matmul_kernel.py:390-424).
Tensors only provide device pointers, strides and the stream; the work is done
by the sm_100a kernels behind the C ABI.
"""

from __future__ import annotations

import ctypes
import threading

import torch

from . import _lib
from ._lib import B2GError, check, lib

_OUT_DT = {torch.float16: _lib.DT_F16, torch.bfloat16: _lib.DT_BF16}
_IN_DT = {torch.float16: _lib.DT_F16, torch.bfloat16: _lib.DT_BF16, torch.float32: _lib.DT_F32}

_ws_lock = threading.Lock()
_workspaces: dict[tuple[int, int], torch.Tensor] = {}
_status: dict[int, torch.Tensor] = {}


def _stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*ts: torch.Tensor) -> torch.device:
    dev = ts[0].device
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("b2g kernels take CUDA tensors (there is no CPU path)")
        if t.device != dev:
            raise ValueError("all operands must be on the same device")
    return dev


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    """Zero-initialised scratch of at least ``nbytes`` for (device, current stream).

    The kernels leave it zeroed after a successful run, so it is reused as is.
    """
    key = (device.index, _stream_handle(device))
    with _ws_lock:
        ws = _workspaces.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
            _workspaces[key] = ws
        return ws


def status_tensor(device: torch.device) -> torch.Tensor:
    """The device status word that kernels on ``device`` report bounded-wait timeouts in."""
    with _ws_lock:
        st = _status.get(device.index)
        if st is None:
            st = torch.zeros(1, dtype=torch.int32, device=device)
            _status[device.index] = st
        return st


def check_status(device: torch.device | None = None, reset: bool = True) -> None:
    """Synchronises ``device`` and raises B2GError if a kernel set the status word.

    After a timeout the stream-K flags in the workspaces may be stale, so they are
    cleared before raising.
    """
    device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    st = status_tensor(device)
    code = int(st.item())
    if code != 0:
        # GEMMs still running on other streams use their workspaces' flags and
        # partial sums: let every stream of the device finish before clearing
        torch.cuda.synchronize(device)
        with _ws_lock:
            for (idx, _), ws in _workspaces.items():
                if idx == device.index:
                    ws.zero_()
        if reset:
            st.zero_()
        torch.cuda.synchronize(device)
        raise B2GError(code, "kernel status")


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _k_major(t: torch.Tensor) -> torch.Tensor:
    """A view (or copy) with unit stride along the last dim, 16-byte row stride and base."""
    eb = t.element_size()
    ok = (t.dim() == 2 and t.stride(1) == 1 and (t.stride(0) * eb) % 16 == 0
          and t.stride(0) >= t.shape[1] and t.data_ptr() % 16 == 0)
    if ok:
        return t
    rows, cols = t.shape
    pad = (-cols * eb) % 16 // eb
    out = torch.zeros((rows, cols + pad), dtype=t.dtype, device=t.device)
    out[:, :cols].copy_(t)
    return out[:, :cols]


def _out(c: torch.Tensor | None, M: int, N: int, dtype: torch.dtype, device) -> torch.Tensor:
    if c is None:
        c = torch.empty((M, N), dtype=dtype, device=device)
    if c.shape != (M, N) or c.dtype not in _OUT_DT:
        raise ValueError(f"c must be ({M}, {N}) fp16/bf16, got {tuple(c.shape)} {c.dtype}")
    return c


def _c_view(c: torch.Tensor) -> tuple[torch.Tensor, bool]:
    """Returns an output buffer the kernel can store into and whether to copy back."""
    eb = c.element_size()
    if c.stride(1) == 1 and (c.stride(0) * eb) % 16 == 0 and c.data_ptr() % 16 == 0:
        return c, False
    return _k_major(torch.empty_like(c)), True


def gemm_f16(a: torch.Tensor, b_t: torch.Tensor, c: torch.Tensor | None = None,
             out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """C = A @ B_t^T for fp16/bf16 A (M, K) and B_t (N, K); C (M, N) fp16/bf16."""
    dev = _require_cuda(a, b_t)
    if a.dtype not in (torch.float16, torch.bfloat16) or b_t.dtype != a.dtype:
        raise ValueError(f"a16w16 takes two fp16 or two bf16 operands, got {a.dtype}, {b_t.dtype}")
    M, K = a.shape
    N, K2 = b_t.shape
    if K != K2:
        raise ValueError("Incompatible dimensions")
    c = _out(c, M, N, out_dtype or (c.dtype if c is not None else a.dtype), dev)
    a_, b_ = _k_major(a), _k_major(b_t)
    cv, copy_back = _c_view(c)
    nbytes = lib().b2g_gemm_workspace_bytes(
        _lib.KIND_F16 if a.dtype == torch.float16 else _lib.KIND_BF16, M, N, K)
    ws = workspace(nbytes, dev)
    rc = lib().b2g_gemm_f16(a_.data_ptr(), a_.stride(0), b_.data_ptr(), b_.stride(0),
                            cv.data_ptr(), cv.stride(0), M, N, K, _IN_DT[a.dtype],
                            _OUT_DT[c.dtype], ws.data_ptr(), ws.numel(),
                            status_tensor(dev).data_ptr(), _stream_handle(dev))
    check(rc, "b2g_gemm_f16")
    if copy_back:
        c.copy_(cv)
    return c


def _as_bytes(t: torch.Tensor) -> torch.Tensor:
    return t if t.dtype == torch.uint8 else t.view(torch.uint8)


def gemm_f8(a: torch.Tensor, b_t: torch.Tensor, c: torch.Tensor | None = None,
            a_scales: torch.Tensor | None = None, b_scales: torch.Tensor | None = None,
            out_dtype: torch.dtype = torch.float16) -> torch.Tensor:
    """C = A @ B_t^T for e5m2 A (M, K), B_t (N, K), optionally with E8M0 scales
    a_scales (M, K/32) and b_scales (N, K/32) of any strides."""
    dev = _require_cuda(a, b_t)
    for t in (a, b_t):
        if t.dtype not in (torch.float8_e5m2, torch.uint8):
            raise ValueError(f"a8w8 takes float8_e5m2 (or raw uint8) operands, got {t.dtype}")
    if (a_scales is None) != (b_scales is None):
        raise ValueError("give both scale tensors or neither")
    M, K = a.shape
    N, K2 = b_t.shape
    if K != K2:
        raise ValueError("Incompatible dimensions")
    c = _out(c, M, N, c.dtype if c is not None else out_dtype, dev)
    a_, b_ = _k_major(_as_bytes(a)), _k_major(_as_bytes(b_t))
    cv, copy_back = _c_view(c)
    scaled = a_scales is not None
    kind = _lib.KIND_MXE5M2 if scaled else _lib.KIND_E5M2
    sa = _scale_args(a_scales, M, K, "a_scales") if scaled else (None, 0, 0)
    sb = _scale_args(b_scales, N, K, "b_scales") if scaled else (None, 0, 0)
    ws = workspace(lib().b2g_gemm_workspace_bytes(kind, M, N, K), dev)
    rc = lib().b2g_gemm_f8(
        a_.data_ptr(), a_.stride(0), b_.data_ptr(), b_.stride(0), *sa, *sb,
        cv.data_ptr(), cv.stride(0), M, N, K, _OUT_DT[c.dtype], ws.data_ptr(), ws.numel(),
        status_tensor(dev).data_ptr(), _stream_handle(dev))
    check(rc, "b2g_gemm_f8")
    if copy_back:
        c.copy_(cv)
    return c


class BlockedScales:
    """E8M0 scales already in the GEMM's blocked layout (see ``block_scales``).

    Passing these instead of a (rows, K/32) tensor skips the per-call relayout,
    which is worth it for static operands such as weights."""

    def __init__(self, data: torch.Tensor, rows: int, K: int):
        self.data, self.rows, self.K = data, rows, K

    @property
    def is_cuda(self) -> bool:
        return self.data.is_cuda

    @property
    def device(self) -> torch.device:
        return self.data.device


def block_scales(s: torch.Tensor, K: int | None = None) -> BlockedScales:
    """(rows, K/32) E8M0 scales of any strides -> BlockedScales (one launch)."""
    dev = _require_cuda(s)
    rows, kb = s.shape
    K = K if K is not None else kb * 32
    out = torch.empty(lib().b2g_scales_blocked_bytes(rows, K), dtype=torch.uint8, device=dev)
    check(lib().b2g_scales_to_blocked(s.data_ptr(), s.stride(0), s.stride(1), rows, K,
                                      out.data_ptr(), _stream_handle(dev)),
          "b2g_scales_to_blocked")
    return BlockedScales(out, rows, K)


def _scale_args(s, rows: int, K: int, name: str) -> tuple[int, int, int]:
    """(pointer, s0, s1) for a scale operand; blocked scales pass strides (0, 0)."""
    if isinstance(s, BlockedScales):
        if (s.rows, s.K) != (rows, K):
            raise ValueError(f"{name} was blocked for ({s.rows}, K={s.K}), need ({rows}, K={K})")
        return s.data.data_ptr(), 0, 0
    _check_scales(s, rows, K, name)
    return s.data_ptr(), s.stride(0), s.stride(1)


def _check_scales(s: torch.Tensor, rows: int, K: int, name: str) -> None:
    if isinstance(s, BlockedScales):
        return
    if s.dtype != torch.uint8 or not s.is_cuda:
        raise ValueError(f"{name} must be a CUDA uint8 (E8M0) tensor")
    if tuple(s.shape) != (rows, K // 32):
        raise ValueError(f"{name} must have shape ({rows}, {K // 32}), got {tuple(s.shape)}")


def gemm_mxf4(a: torch.Tensor, b_t: torch.Tensor, a_scales: torch.Tensor,
              b_scales: torch.Tensor, c: torch.Tensor | None = None,
              out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """C = dequant(A) @ dequant(B_t)^T for packed e2m1 A (M, K/2), B_t (N, K/2)
    and E8M0 scales a_scales (M, K/32), b_scales (N, K/32) of any strides."""
    dev = _require_cuda(a, b_t)
    if a.dtype != torch.uint8 or b_t.dtype != torch.uint8:
        raise ValueError("a4w4 operands are packed uint8")
    M, Kp = a.shape
    N, Kp2 = b_t.shape
    if Kp != Kp2:
        raise ValueError("Incompatible dimensions")
    K = 2 * Kp
    sa = _scale_args(a_scales, M, K, "a_scales")
    sb = _scale_args(b_scales, N, K, "b_scales")
    c = _out(c, M, N, c.dtype if c is not None else out_dtype, dev)
    a_, b_ = _k_major(a), _k_major(b_t)
    cv, copy_back = _c_view(c)
    ws = workspace(lib().b2g_gemm_workspace_bytes(_lib.KIND_MXFP4, M, N, K), dev)
    rc = lib().b2g_gemm_mxf4(
        a_.data_ptr(), a_.stride(0), b_.data_ptr(), b_.stride(0), *sa, *sb,
        cv.data_ptr(), cv.stride(0), M, N, K, _OUT_DT[c.dtype], ws.data_ptr(), ws.numel(),
        status_tensor(dev).data_ptr(), _stream_handle(dev))
    check(rc, "b2g_gemm_mxf4")
    if copy_back:
        c.copy_(cv)
    return c


def gemm_mxf4_grouped(a: torch.Tensor, b_experts: torch.Tensor, a_scales: torch.Tensor,
                      b_scales, group_offsets: torch.Tensor, c: torch.Tensor | None = None,
                      out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """MoE grouped a4w4: rows [g[e], g[e+1]) of A and C use expert e's weights.

    a (M, K/2) packed e2m1, tokens sorted by expert with each expert's segment
    padded to a multiple of 256 rows (128 with the pair option off);
    b_experts (E, N, K/2) or (E * N, K/2); scales (M, K/32) and (E * N, K/32)
    of any strides (or BlockedScales for the experts); group_offsets an int32
    CUDA tensor of E + 1 row offsets (0 first, M last). Returns C (M, N)."""
    dev = _require_cuda(a, b_experts, group_offsets)
    if a.dtype != torch.uint8 or b_experts.dtype != torch.uint8:
        raise ValueError("a4w4 operands are packed uint8")
    if group_offsets.dtype != torch.int32 or group_offsets.dim() != 1:
        raise ValueError("group_offsets must be a 1-D int32 tensor")
    E = group_offsets.numel() - 1
    if E < 1:
        raise ValueError("need at least one group")
    M, Kp = a.shape
    if b_experts.dim() == 3:
        if b_experts.shape[0] != E:
            raise ValueError("b_experts has a different expert count than group_offsets")
        b_experts = b_experts.reshape(-1, b_experts.shape[-1])
    rows_b, Kp2 = b_experts.shape
    if Kp != Kp2 or rows_b % E != 0:
        raise ValueError("Incompatible dimensions")
    N, K = rows_b // E, 2 * Kp
    sa = _scale_args(a_scales, M, K, "a_scales")
    sb = _scale_args(b_scales, rows_b, K, "b_scales")
    c = _out(c, M, N, c.dtype if c is not None else out_dtype, dev)
    a_, b_ = _k_major(a), _k_major(b_experts)
    offs = group_offsets.contiguous()
    cv, copy_back = _c_view(c)
    ws = workspace(lib().b2g_gemm_grouped_workspace_bytes(M, N, K, E), dev)
    rc = lib().b2g_gemm_mxf4_grouped(
        a_.data_ptr(), a_.stride(0), b_.data_ptr(), b_.stride(0), *sa, *sb,
        cv.data_ptr(), cv.stride(0), offs.data_ptr(), E, M, N, K, _OUT_DT[c.dtype],
        ws.data_ptr(), ws.numel(), status_tensor(dev).data_ptr(), _stream_handle(dev))
    check(rc, "b2g_gemm_mxf4_grouped")
    if copy_back:
        c.copy_(cv)
    return c


# ------------------------------------------------------------------ packing --
def quantize_mxfp4(x: torch.Tensor, rows_pad: int | None = None
                   ) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 (rows, K) -> (packed e2m1 (rows, K/2) uint8, E8M0 scales (rows, K/32)).

    The scales are returned as the reference stores them: a (K/32, rows_pad)
    M-contiguous buffer viewed transposed, strides (1, rows_pad)
    (kernels/gemm/intra_wave/a4w4/bench.py:138-144).
    """
    dev = _require_cuda(x)
    if x.dtype != torch.float32 or x.dim() != 2:
        raise ValueError("quantize_mxfp4 takes a 2-D fp32 tensor")
    x = _k_major(x)
    rows, K = x.shape
    rows_pad = rows_pad or rows
    q = torch.empty((rows, K // 2), dtype=torch.uint8, device=dev)
    sc_store = torch.empty((K // 32, rows_pad), dtype=torch.uint8, device=dev)
    sc = sc_store.T[:rows]
    rc = lib().b2g_quant_mxfp4(x.data_ptr(), x.stride(0), rows, K, q.data_ptr(), q.stride(0),
                               sc.data_ptr(), sc.stride(0), sc.stride(1), _stream_handle(dev))
    check(rc, "b2g_quant_mxfp4")
    return q, sc


def quantize_mxe5m2(x: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """fp32 (rows, K) with given E8M0 scales (rows, K/32) -> e5m2 (rows, K)."""
    dev = _require_cuda(x, scales)
    if x.dtype != torch.float32 or x.dim() != 2:
        raise ValueError("quantize_mxe5m2 takes a 2-D fp32 tensor")
    x = _k_major(x)
    rows, K = x.shape
    _check_scales(scales, rows, K, "scales")
    q = torch.empty((rows, K), dtype=torch.uint8, device=dev)
    rc = lib().b2g_quant_mxe5m2(x.data_ptr(), x.stride(0), rows, K, scales.data_ptr(),
                                scales.stride(0), scales.stride(1), q.data_ptr(), q.stride(0),
                                _stream_handle(dev))
    check(rc, "b2g_quant_mxe5m2")
    return q.view(torch.float8_e5m2)


def cast_e5m2(x: torch.Tensor) -> torch.Tensor:
    """Elementwise fp16/bf16/fp32 -> float8_e5m2 with torch's rounding."""
    dev = _require_cuda(x)
    if x.dtype not in _IN_DT:
        raise ValueError(f"cast_e5m2 takes fp16/bf16/fp32, got {x.dtype}")
    xc = x.contiguous()
    out = torch.empty(x.shape, dtype=torch.uint8, device=dev)
    rc = lib().b2g_cast_e5m2(xc.data_ptr(), _IN_DT[x.dtype], xc.numel(), out.data_ptr(),
                             _stream_handle(dev))
    check(rc, "b2g_cast_e5m2")
    return out.view(torch.float8_e5m2)


def plan(kind: int, M: int, N: int, K: int, num_sms: int = 148) -> dict:
    """Host-side schedule summary (no GPU needed)."""
    out = (ctypes.c_int32 * 11)()
    check(lib().b2g_plan_query(kind, M, N, K, num_sms, out, 11), "b2g_plan_query")
    keys = ("cta_group", "tiles_m", "tiles_n", "k_iters", "units", "dp_tiles", "sk_units",
            "launched", "group_m", "splits", "half")
    return dict(zip(keys, list(out)))


def plan_items(kind: int, M: int, N: int, K: int, unit: int, num_sms: int = 148) -> list[tuple]:
    """Work items (tile, tm, tn, k_begin, k_end, role, first_contrib, n_contrib,
    contrib_stride, nh, pair_half) of one unit; nh is -1 for a whole tile, 0 / 1
    for the first / second 128 columns of a half-width tile; pair_half is the
    column half a piece of a two-piece split tile reduces (role 3), else -1."""
    n = lib().b2g_plan_items(kind, M, N, K, num_sms, unit, None, 0)
    if n < 0:
        check(n, "b2g_plan_items")
    buf = (ctypes.c_int32 * (11 * max(n, 1)))()
    lib().b2g_plan_items(kind, M, N, K, num_sms, unit, buf, n)
    return [tuple(buf[11 * i:11 * i + 11]) for i in range(n)]


class PreparedGemm:
    """One GEMM call planned once and launched with nothing but the launch.

    The counterpart of the reference's PreparedKernel (scripts/prepared_kernel.py:
    76-138), which binds a launch's arguments once so that back-to-back calls pay
    no launcher overhead (scripts/benchmark_prepared.py:255-260). Preparation
    checks the operands, fixes the schedule under the current options and encodes
    every tensor map (b2g_prepare_gemm); each call then launches on the current
    stream (b2g_prepared_run) and returns C. The operands, scales and C stay
    referenced: their contents may change between calls, their storage may not.
    The call owns its workspace, so it can run on any stream, but two calls of
    the same object must not overlap on the GPU. Build one with prepare_gemm_f16,
    prepare_gemm_f8 or prepare_gemm_mxf4."""

    def __init__(self, kind: int, a_: torch.Tensor, b_: torch.Tensor, sa: tuple, sb: tuple,
                 c: torch.Tensor, M: int, N: int, K: int, keep: tuple):
        dev = c.device
        self.device, self.c = dev, c
        self._keep = (a_, b_, c) + keep
        # a zeroed workspace of its own (its flag words must read zero at rest)
        self._ws = torch.zeros(max(lib().b2g_gemm_workspace_bytes(kind, M, N, K), 256),
                               dtype=torch.uint8, device=dev)
        self._h = ctypes.c_void_p()
        rc = lib().b2g_prepare_gemm(kind, a_.data_ptr(), a_.stride(0), b_.data_ptr(),
                                    b_.stride(0), *sa, *sb, c.data_ptr(), c.stride(0), M, N, K,
                                    _OUT_DT[c.dtype], self._ws.data_ptr(), self._ws.numel(),
                                    status_tensor(dev).data_ptr(), ctypes.byref(self._h))
        check(rc, "b2g_prepare_gemm")

    def __call__(self) -> torch.Tensor:
        if not self._h:
            raise B2GError(_lib.EINVAL, "prepared GEMM already closed")
        check(lib().b2g_prepared_run(self._h, _stream_handle(self.device)), "b2g_prepared_run")
        return self.c

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().b2g_prepared_free(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:  # interpreter shutdown: the library may be gone
            pass


def _in_place(t: torch.Tensor, name: str) -> torch.Tensor:
    """The operand itself when the kernel can read it where it lies (a prepared
    call keeps reading that storage, so a padded copy would go stale)."""
    if _k_major(t) is not t:
        raise ValueError(f"a prepared GEMM reads {name} in place: give it K-contiguous with "
                         "16-byte aligned base and rows")
    return t


def _prepared_c(c: torch.Tensor | None, M: int, N: int, dtype: torch.dtype, dev) -> torch.Tensor:
    c = _out(c, M, N, dtype, dev)
    if _c_view(c)[1]:
        raise ValueError("a prepared GEMM stores straight into C: give a C with unit column "
                         "stride and 16-byte aligned rows")
    return c


def prepare_gemm_f16(a: torch.Tensor, b_t: torch.Tensor, c: torch.Tensor | None = None,
                     out_dtype: torch.dtype | None = None) -> PreparedGemm:
    """gemm_f16(a, b_t, c) as a PreparedGemm (same operand rules)."""
    dev = _require_cuda(a, b_t)
    if a.dtype not in (torch.float16, torch.bfloat16) or b_t.dtype != a.dtype:
        raise ValueError(f"a16w16 takes two fp16 or two bf16 operands, got {a.dtype}, {b_t.dtype}")
    M, K = a.shape
    N, K2 = b_t.shape
    if K != K2:
        raise ValueError("Incompatible dimensions")
    c = _prepared_c(c, M, N, out_dtype or (c.dtype if c is not None else a.dtype), dev)
    kind = _lib.KIND_F16 if a.dtype == torch.float16 else _lib.KIND_BF16
    return PreparedGemm(kind, _in_place(a, "a"), _in_place(b_t, "b_t"), (None, 0, 0),
                        (None, 0, 0), c, M, N, K, ())


def prepare_gemm_f8(a: torch.Tensor, b_t: torch.Tensor, c: torch.Tensor | None = None,
                    a_scales=None, b_scales=None,
                    out_dtype: torch.dtype = torch.float16) -> PreparedGemm:
    """gemm_f8(a, b_t, c, a_scales, b_scales) as a PreparedGemm (same operand rules)."""
    dev = _require_cuda(a, b_t)
    for t in (a, b_t):
        if t.dtype not in (torch.float8_e5m2, torch.uint8):
            raise ValueError(f"a8w8 takes float8_e5m2 (or raw uint8) operands, got {t.dtype}")
    if (a_scales is None) != (b_scales is None):
        raise ValueError("give both scale tensors or neither")
    M, K = a.shape
    N, K2 = b_t.shape
    if K != K2:
        raise ValueError("Incompatible dimensions")
    c = _prepared_c(c, M, N, c.dtype if c is not None else out_dtype, dev)
    scaled = a_scales is not None
    sa = _scale_args(a_scales, M, K, "a_scales") if scaled else (None, 0, 0)
    sb = _scale_args(b_scales, N, K, "b_scales") if scaled else (None, 0, 0)
    kind = _lib.KIND_MXE5M2 if scaled else _lib.KIND_E5M2
    return PreparedGemm(kind, _in_place(_as_bytes(a), "a"), _in_place(_as_bytes(b_t), "b_t"), sa,
                        sb, c, M, N, K, (a_scales, b_scales))


def prepare_gemm_mxf4(a: torch.Tensor, b_t: torch.Tensor, a_scales, b_scales,
                      c: torch.Tensor | None = None,
                      out_dtype: torch.dtype = torch.bfloat16) -> PreparedGemm:
    """gemm_mxf4(a, b_t, a_scales, b_scales, c) as a PreparedGemm (same operand rules)."""
    dev = _require_cuda(a, b_t)
    if a.dtype != torch.uint8 or b_t.dtype != torch.uint8:
        raise ValueError("a4w4 operands are packed uint8")
    M, Kp = a.shape
    N, Kp2 = b_t.shape
    if Kp != Kp2:
        raise ValueError("Incompatible dimensions")
    K = 2 * Kp
    sa = _scale_args(a_scales, M, K, "a_scales")
    sb = _scale_args(b_scales, N, K, "b_scales")
    c = _prepared_c(c, M, N, c.dtype if c is not None else out_dtype, dev)
    return PreparedGemm(_lib.KIND_MXFP4, _in_place(a, "a"), _in_place(b_t, "b_t"), sa, sb, c,
                        M, N, K, (a_scales, b_scales))


__all__ = [
    "B2GError", "BlockedScales", "block_scales", "gemm_f16", "gemm_f8", "gemm_mxf4",
    "quantize_mxfp4", "quantize_mxe5m2",
    "cast_e5m2", "workspace", "status_tensor", "check_status", "plan", "plan_items",
    "PreparedGemm", "prepare_gemm_f16", "prepare_gemm_f8", "prepare_gemm_mxf4",
]
