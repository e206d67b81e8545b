"""Drop-in for the reference's FMHA forward launcher.

Mirrors ``run_gluon_attention(q, k, v, o, metadata, scale_on_q=True)`` of
kernels/attention/fmha_v4.py:761-790 and the host helpers it reads from
kernels/attention/common.py (``MetaData`` :58-69, ``get_shape_from_layout``
:72-81, ``get_strides_from_layout`` :84-92, ``input_helper`` :95-112,
``compute_flops`` :177-184): same argument meaning, the same ``bhsd`` / ``bshd``
layouts, output written into ``o`` on the current stream. The work runs in
the sm_100a flash-attention kernel of libb2g.so (``b2g_attention_fwd``).

Differences from the reference launcher, all widenings: Q and K lengths may
differ and need not be multiples of 64 (rows and keys past the ends are
masked), and the softmax log-sum-exp can be returned. ``scale_on_q`` is
accepted for signature compatibility; the kernel always applies the scale to
the fp32 scores, which is the more accurate of the reference's two choices.
Causal masking is not supported, as in the reference tutorial kernel.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _lib
from .ops import _require_cuda, _stream_handle, status_tensor

_DT = {torch.float16: _lib.DT_F16, torch.bfloat16: _lib.DT_BF16}
HEAD_DIMS = (64, 128)
BLOCK_M, BLOCK_N = 128, 128   # query rows per CTA, keys per tile
KERNEL_NAME = "fmha_fwd_kernel"


class MetaData:
    """Host-side descriptor of one attention problem (fields of common.py:58-69)."""

    causal = False
    layout = None
    max_seqlens_q = 0
    max_seqlens_k = 0

    def __init__(self, sm_scale: float = 1.0):
        self.sm_scale = sm_scale


def get_shape_from_layout(q: torch.Tensor, k: torch.Tensor, metadata: MetaData):
    """(batch, heads_q, heads_k, head_dim) of a ``bhsd`` or ``bshd`` problem."""
    if metadata.layout == "bhsd":
        return q.shape[0], q.shape[1], k.shape[1], q.shape[3]
    if metadata.layout == "bshd":
        return q.shape[0], q.shape[2], k.shape[2], q.shape[3]
    raise ValueError(f"Unsupported layout: {metadata.layout}")


def _axis_order(layout: str) -> tuple[int, int, int, int]:
    if layout == "bhsd":
        return (0, 1, 2, 3)
    if layout == "bshd":
        return (0, 2, 1, 3)
    raise ValueError(f"Unsupported layout: {layout}")


def get_strides_from_layout(q, k, v, o, metadata: MetaData):
    """Each tensor's strides in (batch, head, sequence, dim) order."""
    order = _axis_order(metadata.layout)
    return tuple(tuple(t.stride(i) for i in order) for t in (q, k, v, o))


def input_helper(Z, HQ, HK, N_CTX_Q, N_CTX_K, D_HEAD, dtype, layout, requires_grad=False,
                 device="cuda"):
    """Seeded standard-normal q, k, v in ``layout`` and their MetaData, the
    problem recipe of the reference's bench (seed 20, sm_scale = D ** -0.5)."""
    if layout not in ("bhsd", "bshd"):
        raise ValueError(f"Unsupported layout: {layout}")
    torch.manual_seed(20)

    def rand(heads, n_ctx):
        shape = (Z, heads, n_ctx, D_HEAD) if layout == "bhsd" else (Z, n_ctx, heads, D_HEAD)
        return torch.randn(shape, dtype=dtype, device=device, requires_grad=requires_grad)

    q = rand(HQ, N_CTX_Q)
    k = rand(HK, N_CTX_K)
    v = rand(HK, N_CTX_K)
    md = MetaData(sm_scale=D_HEAD ** -0.5)
    md.max_seqlens_q = N_CTX_Q
    md.max_seqlens_k = N_CTX_K
    md.layout = layout
    return q, k, v, md


def compute_flops(B, HQ, M, N, D, causal=False):
    """FLOPs of the forward pass: the QK^T and PV products, 2*B*HQ*M*N*D each."""
    if causal:
        valid = ((N ** 2 + N) / 2) if M > N else (M * N - ((M ** 2 - M) / 2))
        per_matmul = 2.0 * B * HQ * valid * D
    else:
        per_matmul = 2.0 * B * HQ * M * N * D
    return 2 * per_matmul


def attention_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                  o: torch.Tensor | None = None, *, sm_scale: float | None = None,
                  layout: str = "bhsd", lse: torch.Tensor | None = None) -> torch.Tensor:
    """O = softmax(Q K^T * sm_scale) V per (batch, query head), GQA by head groups.

    ``q`` is (B, HQ, Sq, D) for ``bhsd`` or (B, Sq, HQ, D) for ``bshd``; ``k`` and
    ``v`` likewise with HK heads and Sk keys; ``o`` takes q's shape and dtype.
    ``lse``, if given, is a float32 (B, HQ, Sq) tensor that receives the
    natural-log log-sum-exp of each row's scaled scores. Asynchronous on the
    current stream; kernel timeouts are reported by ``ops.check_status``.
    """
    dev = _require_cuda(q, k, v, o, lse)
    order = _axis_order(layout)
    if q.dtype not in _DT or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("q, k and v must share one dtype, float16 or bfloat16")
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError("q, k and v must be 4-D")
    B, HQ, Sq, D = (q.shape[i] for i in order)
    Bk, HK, Sk, Dk = (k.shape[i] for i in order)
    if (Bk, Dk) != (B, D) or tuple(v.shape) != tuple(k.shape):
        raise ValueError(f"k/v shapes {tuple(k.shape)}/{tuple(v.shape)} do not match q {tuple(q.shape)}")
    if o is None:
        o = torch.empty_like(q)
    if tuple(o.shape) != tuple(q.shape) or o.dtype != q.dtype:
        raise ValueError("o must have q's shape and dtype")
    if lse is not None and (lse.dtype != torch.float32 or tuple(lse.shape) != (B, HQ, Sq)
                            or not lse.is_contiguous()):
        raise ValueError(f"lse must be a contiguous float32 ({B}, {HQ}, {Sq}) tensor")
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)

    ts = []
    for t in (q, k, v):
        if t.stride(order[3]) != 1 or any((t.stride(i) * 2) % 16 for i in order[:3]) \
                or t.data_ptr() % 16:
            t = t.contiguous()
        ts.append(t)
    o_run = o
    if o.stride(order[3]) != 1 or any((o.stride(i) * 2) % 16 for i in order[:3]) \
            or o.data_ptr() % 16:
        o_run = torch.empty_like(q, memory_format=torch.contiguous_format)
    strides = (ctypes.c_int64 * 16)(*[t.stride(i) for t in (*ts, o_run) for i in order])
    st = status_tensor(dev)
    rc = _lib.lib().b2g_attention_fwd(
        ts[0].data_ptr(), ts[1].data_ptr(), ts[2].data_ptr(), o_run.data_ptr(), strides,
        B, HQ, HK, Sq, Sk, D, _DT[q.dtype], float(sm_scale),
        None if lse is None else lse.data_ptr(), st.data_ptr(), _stream_handle(dev))
    _lib.check(rc)
    if o_run is not o:
        o.copy_(o_run)
    return o


def run_gluon_attention(q, k, v, o, metadata: MetaData, scale_on_q: bool = True):
    """Runs the forward pass on ``q, k, v`` and writes the result into ``o``.

    Same contract as the reference launcher: non-causal only, ``metadata.layout``
    ``bhsd`` or ``bshd``, ``metadata.sm_scale`` the softmax scale. Head dims 64
    and 128 (the reference takes any power of two).
    """
    assert not metadata.causal, "the FMHA forward kernel supports non-causal attention only"
    batch, nheads_q, nheads_k, head_size = get_shape_from_layout(q, k, metadata)
    assert head_size & (head_size - 1) == 0, "head dim must be a power of two"
    assert head_size in HEAD_DIMS, f"head dim must be one of {HEAD_DIMS}"
    assert nheads_q % nheads_k == 0, "query heads must be a multiple of key/value heads"
    del scale_on_q  # the scale is always applied to the fp32 scores
    return attention_fwd(q, k, v, o, sm_scale=metadata.sm_scale, layout=metadata.layout)


def main(argv=None) -> None:
    """Times the forward pass on one problem, with the reference FMHA bench's
    flags and defaults (kernels/attention/bench.py:103-155): seeded inputs,
    CUDA-event timing on the current stream, TFLOPS from compute_flops."""
    import argparse

    ap = argparse.ArgumentParser(description="B200 FMHA forward timing")
    ap.add_argument("--dtype", choices=["fp16", "bf16"], default="bf16")
    ap.add_argument("--layout", choices=["bhsd", "bshd"], default="bhsd")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--hq", type=int, default=64)
    ap.add_argument("--hk", type=int, default=64)
    ap.add_argument("--d", type=int, default=128)
    ap.add_argument("--seqlen", type=int, default=8192)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=10)
    args = ap.parse_args(argv)
    from .ops import check_status

    dt = torch.bfloat16 if args.dtype == "bf16" else torch.float16
    q, k, v, md = input_helper(args.batch, args.hq, args.hk, args.seqlen, args.seqlen, args.d, dt,
                               args.layout)
    o = torch.empty_like(q)
    for _ in range(args.warmup):
        run_gluon_attention(q, k, v, o, md)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.iters):
        run_gluon_attention(q, k, v, o, md)
    end.record()
    torch.cuda.synchronize()
    check_status()
    ms = start.elapsed_time(end) / max(args.iters, 1)
    flops = compute_flops(args.batch, args.hq, args.seqlen, args.seqlen, args.d, False)
    print(f"FMHA B={args.batch} HQ={args.hq} HK={args.hk} S={args.seqlen} D={args.d} "
          f"{args.dtype} {args.layout}: {ms * 1e3:.1f} us, {flops / ms / 1e9:.1f} TFLOPS")


if __name__ == "__main__":
    main()
