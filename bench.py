"""Benchmark driver for the B200 GEMM hot path.

Default (driver contract):  python bench.py [--gpus N] [--steps K] [--warmup W]
  One process per GPU (torchrun for N > 1). The headline workload is BASELINE
  a16w16 FP16 C = A @ B^T with M = 4096, K = 8192 and 4096 columns of
  C per GPU - B is sharded along N across the ranks (A replicated, no collective
  in the timed loop), so per-GPU work is fixed as N grows ("weak" scaling).
  The same line carries the BF8 and MXFP4 rates at
  the same shape, a roofline object for the GEMM kernel, the CPU baseline, an
  end-to-end number through the public API with host buffers, the clocks seen
  while timing and (N > 1) a separately timed NCCL all-gather of the C slabs.

  --impl reference   times the reference's CPU path for the same workload
                     (torch.matmul in fp16 on the host cores - the oracle's
                     restatement of kernels/gemm/intra_wave/a16w16/bench.py:183).
  --config large     BASELINE configs[4]: MXFP4 16384 x 53248 x 16384 with N
                     split over the ranks (fixed total work: "strong" scaling).

Reference bench surface (kernels/gemm/intra_wave/<kind>/bench.py:133-164):
  python bench.py --kernel a16w16|a8w8|a4w4 [--K 8192] [--dtype fp16 bf16]
                  [--M 4096 --N 4096] [--rocprof] [--rotating-buffer-size 512]
                  [--prepared]
  runs the correctness check against torch on the GPU and prints the TFLOPS
  table, or with --rocprof 1000 launches over rotating buffers for an external
  profiler (ncu here). --prepared times prepared calls (ops.PreparedGemm,
  planned once and then only launched), as scripts/benchmark_prepared.py does.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
PEAKS_PATH = os.path.join(ROOT, "MEASURED_PEAKS.json")
TRAFFIC_PATH = os.path.join(ROOT, "profiles", "traffic.json")
METRIC = "GEMM TFLOPS/GPU & % of dtype dense peak (FP16, BF8, MXFP4) at 1/2/4/8 B200"
NOMINAL_DENSE_TFLOPS = {"fp16": 2250.0, "bf16": 2250.0, "bf8": 4500.0, "mxfp4": 9000.0}
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


# ----------------------------------------------------------------- helpers --
def log(*a):
    print(*a, file=sys.stderr, flush=True)


def load_peaks() -> tuple[dict, str]:
    try:
        with open(PEAKS_PATH) as f:
            return json.load(f), "measured"
    except (OSError, ValueError):
        return dict(FALLBACK_PEAKS), "fallback"


def tensor_peak(dtype_name: str, peaks: dict) -> float:
    """Dense peak for a dtype: the measured bf16 GEMM rate scaled by the
    hardware's dtype ratio (fp8 2x, fp4 4x of fp16/bf16)."""
    mult = {"fp16": 1.0, "bf16": 1.0, "bf8": 2.0, "mxfp4": 4.0}[dtype_name]
    return peaks["bf16_tflops"] * mult


class ClockSampler:
    """SM clock and throttle reasons sampled while timing.

    Polls NVML from a background thread about every millisecond (the timed
    region of a default run is only tens of ms); reports the absence when the
    NVML bindings are missing."""

    REASONS = {  # NVML clocks-event reason bits reported as rejection criteria
        "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
        "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, index: int):
        self.index = index
        self.samples: list[tuple[float, float, int, float]] = []
        self._stop = threading.Event()
        self.thread = None
        self.nvml = None

    def start(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            self.handle = pynvml.nvmlDeviceGetHandleByIndex(self._physical_index())
        except Exception:  # noqa: BLE001 - no NVML: report the absence
            self.nvml = None
            return
        self.thread = threading.Thread(target=self._poll, daemon=True)
        self.thread.start()

    def _physical_index(self) -> int:
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        if vis:
            try:
                return int(vis.split(",")[self.index])
            except (ValueError, IndexError):
                pass
        return self.index

    def _poll(self):
        n = self.nvml
        try:
            smax = float(n.nvmlDeviceGetMaxClockInfo(self.handle, n.NVML_CLOCK_SM))
        except Exception:  # noqa: BLE001
            return
        power, i = 0.0, 0
        while not self._stop.is_set():
            try:
                sm = n.nvmlDeviceGetClockInfo(self.handle, n.NVML_CLOCK_SM)
                reasons = n.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                if i % 5 == 0:  # the power reading is the slowest query
                    power = n.nvmlDeviceGetPowerUsage(self.handle) / 1000.0
                self.samples.append((float(sm), smax, int(reasons), power, time.perf_counter()))
            except Exception:  # noqa: BLE001
                break
            i += 1
            time.sleep(0.0005)

    def stop(self, window: tuple[float, float] | None = None) -> dict:
        """Summary of the samples taken inside `window` (host perf_counter times
        bracketing the timed region), or of all samples if none fall inside."""
        if self.nvml is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        self._stop.set()
        if self.thread is not None:
            self.thread.join(timeout=2)
        sel = self.samples
        if window is not None:
            inside = [x for x in self.samples if window[0] <= x[4] <= window[1]]
            sel = inside or self.samples
        if not sel:
            return {"sm_mhz": None, "sm_max_mhz": None, "samples": 0, "reasons": []}
        sm = [x[0] for x in sel]
        reasons = sorted({name for x in sel for name, bit in self.REASONS.items() if x[2] & bit})
        return {"sm_mhz": statistics.median(sm), "sm_min_mhz": min(sm),
                "sm_max_mhz": max(x[1] for x in sel), "power_w_max": max(x[3] for x in sel),
                "samples": len(sel), "reasons": reasons}


def dist_setup(n_gpus: int, cuda: bool = True):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group(
            "nccl", timeout=datetime.timedelta(seconds=120),
            device_id=torch.device("cuda", local))
    elif cuda:
        torch.cuda.set_device(0)
    if world != n_gpus and rank == 0:
        log(f"note: --gpus {n_gpus} but WORLD_SIZE={world}; using {world}")
    return rank, world, local


def barrier(world: int):
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------- checker --
# Parity of what was timed: after each leg's timed region, seeded 128 x 128
# blocks of its output are recomputed on the CPU by the oracle (the
# reference's dequantise-then-fp32-matmul, restated in oracle/ and pinned to
# the reference's own functions) and compared under the build's tolerances.
# The oracle is only the checker here; nothing it computes is timed.
TOL = {"fp16": 1e-2, "bf16": 1e-2, "bf8": 3e-2, "mxfp4": 3e-2}


def pick_blocks(M: int, N: int, n: int, seed: int, bm: int = 128, bn: int = 128) -> list:
    """n seeded (row, col) origins of bm x bn blocks inside an M x N output."""
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(n):
        r0 = int(torch.randint(0, max(1, (M - bm) // 16 + 1), (1,), generator=g)) * 16
        c0 = int(torch.randint(0, max(1, (N - bn) // 16 + 1), (1,), generator=g)) * 16
        out.append((min(r0, max(0, M - bm)), min(c0, max(0, N - bn))))
    return out


def parity_gemm(kind: str, inp: dict, c: torch.Tensor, blocks: list, b_row0: int = 0) -> dict:
    """Checks blocks of C = A B^T against the oracle. `inp` holds a, b (N x K
    storage) and, for scaled kinds, sa / sb ((rows, K/32) E8M0 of any strides);
    `b_row0` offsets B's rows (a block's columns c0.. use B rows b_row0 + c0..)."""
    import numpy as np
    from oracle import mx
    worst, exact, n_el = 0.0, 0, 0
    for r0, c0 in blocks:
        rs, cs = slice(r0, r0 + 128), slice(b_row0 + c0, b_row0 + c0 + 128)
        got = c[r0:r0 + 128, c0:c0 + 128].contiguous()
        if kind in ("fp16", "bf16"):
            a = inp["a"][rs].contiguous()
            b = inp["b"][cs].contiguous()
            if kind == "fp16":
                ref = mx.gemm_f16_ref(a.cpu().numpy(), b.cpu().numpy()).astype(np.float32)
                g32 = got.float().cpu().numpy()
            else:
                bits = lambda t: t.view(torch.int16).cpu().numpy().view(np.uint16)  # noqa: E731
                ref_bits = mx.gemm_f16_ref(bits(a), bits(b), "bf16")
                ref = mx.bf16_bits_to_f32(ref_bits)
                g32 = got.float().cpu().numpy()
                exact += int(np.sum(bits(got) == ref_bits))
        else:
            a = inp["a"][rs].contiguous().view(torch.uint8).cpu().numpy()
            b = inp["b"][cs].contiguous().view(torch.uint8).cpu().numpy()
            sa = inp["sa"][rs].cpu().numpy()
            sb = inp["sb"][cs].cpu().numpy()
            fn = mx.gemm_mxfp4_ref if kind == "mxfp4" else mx.gemm_mxe5m2_ref
            ref_bits = fn(a, b, sa, sb)
            got_bits = got.view(torch.int16).cpu().numpy().view(np.uint16)
            ref = mx.bf16_bits_to_f32(ref_bits)
            g32 = mx.bf16_bits_to_f32(got_bits)
            exact += int(np.sum(got_bits == ref_bits))
        n_el += got.numel()
        worst = max(worst, mx.normalised_max_abs(g32, ref))
    res = {"ok": bool(worst <= TOL[kind]), "max_norm_err": worst, "tol": TOL[kind],
           "blocks": [list(b) for b in blocks], "checker": "oracle (CPU)"}
    if kind != "fp16":
        res["bit_exact_frac"] = exact / max(1, n_el)
    return res


# --------------------------------------------------------------- workloads --
class Workload:
    """One GEMM configuration with rotating device inputs (cold L2 per step)."""

    def __init__(self, name: str, M: int, N: int, K: int, dtype_name: str, sets: int,
                 seed: int):
        from gfx950_gluon_tutorials_b200 import ops
        self.ops = ops
        self.name, self.M, self.N, self.K, self.dtype_name = name, M, N, K, dtype_name
        self.flops = 2.0 * M * N * K
        dev = torch.device("cuda", torch.cuda.current_device())
        gen = torch.Generator(device=dev).manual_seed(seed)
        self.sets = []
        for _ in range(sets):
            self.sets.append(self._make(gen, dev))
        # scaled kinds: the scale relayout and the GEMM
        self.launches_per_step = 1 if dtype_name in ("fp16", "bf16") else 2

    def _make(self, gen, dev):
        M, N, K = self.M, self.N, self.K
        if self.dtype_name in ("fp16", "bf16"):
            dt = torch.float16 if self.dtype_name == "fp16" else torch.bfloat16
            a = (torch.randn((M, K), generator=gen, device=dev) / K ** 0.5).to(dt)
            b = (torch.randn((N, K), generator=gen, device=dev) / K ** 0.5).to(dt)
            return {"a": a, "b": b, "c": torch.empty((M, N), dtype=dt, device=dev)}
        if self.dtype_name == "bf8":
            out = {}
            for key, rows in (("a", M), ("b", N)):
                x = torch.randn((rows, K), generator=gen, device=dev)
                e = torch.randint(125, 130, (rows, K // 32), generator=gen, device=dev).to(
                    torch.uint8)
                out[key] = self.ops.quantize_mxe5m2(x, e)
                out["s" + key] = e
                del x
            out["c"] = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
            return out
        out = {}
        for key, rows in (("a", M), ("b", N)):
            x = torch.randn((rows, K), generator=gen, device=dev)
            rows_pad = (rows + 255) // 256 * 256
            out[key], out["s" + key] = self.ops.quantize_mxfp4(x, rows_pad=rows_pad)
            del x
        out["c"] = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
        return out

    def run(self, i: int):
        s = self.sets[i % len(self.sets)]
        if self.dtype_name in ("fp16", "bf16"):
            return self.ops.gemm_f16(s["a"], s["b"], s["c"])
        if self.dtype_name == "bf8":
            return self.ops.gemm_f8(s["a"], s["b"], s["c"], a_scales=s["sa"], b_scales=s["sb"])
        return self.ops.gemm_mxf4(s["a"], s["b"], s["sa"], s["sb"], s["c"])

    def check(self, seed: int, n_blocks: int = 2) -> dict:
        """Parity of one more call on input set 0 (outside any timed region)."""
        out = self.run(0)
        torch.cuda.synchronize()
        self.ops.check_status()
        s = self.sets[0]
        inp = {"a": s["a"], "b": s["b"], "sa": s.get("sa"), "sb": s.get("sb")}
        return parity_gemm(self.dtype_name, inp, out, pick_blocks(self.M, self.N, n_blocks, seed))

    def input_bytes(self) -> int:
        s = self.sets[0]
        return sum(t.numel() * t.element_size() for k, t in s.items() if k != "c")

    def set_bytes(self) -> int:
        s = self.sets[0]
        return sum(t.numel() * t.element_size() for t in s.values())


def time_device(w: Workload, steps: int, warmup: int, world: int, marks: list | None = None
                ) -> float:
    """ms per step: CUDA events on the launching stream, max over ranks. `marks`
    receives the host times bracketing the timed region."""
    for i in range(warmup):
        w.run(i)
    barrier(world)
    stream = torch.cuda.current_stream()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    start.record(stream)
    for i in range(steps):
        w.run(warmup + i)
    end.record(stream)
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    if marks is not None:
        marks.extend([t0, t1])
    ms = start.elapsed_time(end) / steps
    barrier(world)
    w.ops.check_status()
    return max_over_ranks(ms, world)


def time_e2e(w: Workload, steps: int, warmup: int, world: int) -> tuple[float, int, int]:
    """Public-API calls on host inputs, as a streaming caller runs them: every
    step copies its own A and B (and scales) from pinned host memory, runs the
    GEMM and copies its C back to pinned host memory. Device inputs and outputs
    are double-buffered, so step i+1's upload and step i-1's download (separate
    streams, PCIe is full duplex) overlap step i's GEMM; events order each
    buffer's reuse. All of it lies inside the timed region."""
    s = w.sets[0]
    host_in = {k: torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for k, t in s.items()
               if k != "c"}
    for k in host_in:
        host_in[k].copy_(s[k])
    host_c = [torch.empty(s["c"].shape, dtype=s["c"].dtype, pin_memory=True) for _ in range(2)]
    dev = [{k: torch.empty_like(s[k]) for k in host_in} for _ in range(2)]
    h2d = sum(t.numel() * t.element_size() for t in host_in.values())
    d2h = host_c[0].numel() * host_c[0].element_size()
    ops = w.ops
    up, comp, down = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    ev = lambda: torch.cuda.Event()
    uploaded, computed, downloaded = [ev(), ev()], [ev(), ev()], [ev(), ev()]
    outs: list = [None, None]

    def matmul(d):
        if w.dtype_name in ("fp16", "bf16"):
            from gfx950_gluon_tutorials_b200 import a16w16
            return a16w16.matmul(d["a"], d["b"].T)
        if w.dtype_name == "bf8":
            from gfx950_gluon_tutorials_b200 import a8w8
            return a8w8.matmul_scaled(d["a"], d["b"].T, d["sa"], d["sb"])
        from gfx950_gluon_tutorials_b200 import a4w4
        return a4w4.matmul(d["a"], d["b"], d["sa"], d["sb"])

    def step(i):
        j = i % 2
        d = dev[j]
        up.wait_event(computed[j])           # the GEMM of step i-2 read these inputs
        with torch.cuda.stream(up):
            for k in host_in:
                d[k].copy_(host_in[k], non_blocking=True)
        uploaded[j].record(up)
        comp.wait_event(uploaded[j])
        comp.wait_event(downloaded[j])       # C of step i-2 has left the device
        with torch.cuda.stream(comp):
            outs[j] = matmul(d)
        computed[j].record(comp)
        down.wait_event(computed[j])
        with torch.cuda.stream(down):
            host_c[j].copy_(outs[j], non_blocking=True)
        downloaded[j].record(down)

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    barrier(world)
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(up)
    comp.wait_stream(up)
    down.wait_stream(up)
    for i in range(steps):
        step(warmup + i)
    down.wait_stream(up)
    down.wait_stream(comp)
    end.record(down)
    torch.cuda.synchronize()
    ms = max_over_ranks(start.elapsed_time(end) / steps, world)
    ops.check_status()
    return ms, h2d, d2h


def time_skinny(world: int, peaks: dict, peak_src: str, iters: int = 20) -> dict:
    """Memory-bound leg: a decode-like C = A * B^T with M = 16 rows of A against
    this rank's N-shard of the large configuration's weight matrix (N = 53248 / g,
    K = 16384, fp16). Runs the small-M swap-AB kernel; the bound is reading B
    once from HBM (B alone is far larger than L2)."""
    from gfx950_gluon_tutorials_b200 import ops
    M, N, K = 16, 53248 // world, 16384
    dev = torch.device("cuda", torch.cuda.current_device())
    gen = torch.Generator(device=dev).manual_seed(77)
    a = (torch.randn((M, K), generator=gen, device=dev) / K ** 0.5).half()
    b = (torch.randn((N, K), generator=gen, device=dev) / K ** 0.5).half()
    c = torch.empty((M, N), dtype=torch.float16, device=dev)
    for _ in range(3):
        ops.gemm_f16(a, b, c)
    barrier(world)
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(iters):
        ops.gemm_f16(a, b, c)
    end.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(start.elapsed_time(end) / iters, world)
    ops.check_status()
    algo = (M * K + N * K + M * N) * 2
    gbs = algo / (ms * 1e-3) / 1e9
    out = {"workload": f"fp16 M={M} N={N} K={K} per GPU (decode against a weight shard)",
           "us_per_call": ms * 1e3, "tflops_per_gpu": 2.0 * M * N * K / (ms * 1e-3) / 1e12,
           "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"],
                        "unit": "GB/s", "frac": gbs / peaks["hbm_gbs"],
                        "algorithmic_bytes_per_launch": algo,
                        "peak_source": f"{peak_src} hbm_gbs (copy)"}}
    del a, b, c
    torch.cuda.empty_cache()
    return out


def time_moe(world: int, peaks: dict, steps: int, warmup: int) -> dict:
    """MoE grouped MXFP4 leg: 8 experts with 1024 tokens routed to each (an
    8192-row A, tokens sorted by expert), expert weights N = 4096 x K = 8192,
    quantised N(0,1) data, expert scales relaid once (static weights)."""
    from gfx950_gluon_tutorials_b200 import a4w4, ops
    E, rows, N, K = 8, 1024, 4096, 8192
    dev = torch.device("cuda", torch.cuda.current_device())
    gen = torch.Generator(device=dev).manual_seed(91)
    qa, sa = ops.quantize_mxfp4(torch.randn((E * rows, K), generator=gen, device=dev))
    qb, sb_rows = ops.quantize_mxfp4(torch.randn((E * N, K), generator=gen, device=dev))
    sb = ops.block_scales(sb_rows, K)
    offs = torch.arange(0, E * rows + 1, rows, dtype=torch.int32, device=dev)
    c = torch.empty((E * rows, N), dtype=torch.bfloat16, device=dev)
    for _ in range(warmup):
        a4w4.grouped_matmul(qa, qb, sa, sb, offs, c=c)
    barrier(world)
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        a4w4.grouped_matmul(qa, qb, sa, sb, offs, c=c)
    end.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(start.elapsed_time(end) / steps, world)
    ops.check_status()
    flops = 2.0 * E * rows * N * K
    tf = flops / (ms * 1e-3) / 1e12
    # parity: a block of two experts' rows against the oracle with that
    # expert's weights (expert e's B rows start at e * N)
    sb_raw = sb_rows
    checks = []
    for e, (r0, c0) in zip((1, E - 2), pick_blocks(rows, N, 2, 911)):
        seg = slice(e * rows, (e + 1) * rows)
        inp = {"a": qa[seg], "b": qb, "sa": sa[seg], "sb": sb_raw}
        checks.append(parity_gemm("mxfp4", inp, c[e * rows:(e + 1) * rows], [(r0, c0)],
                                  b_row0=e * N))
    parity = {"ok": all(x["ok"] for x in checks),
              "max_norm_err": max(x["max_norm_err"] for x in checks), "tol": TOL["mxfp4"],
              "bit_exact_frac": min(x["bit_exact_frac"] for x in checks),
              "blocks": [[e, *x["blocks"][0]] for e, x in zip((1, E - 2), checks)],
              "checker": "oracle (CPU), expert's own weight rows"}
    del qa, qb, sa, sb, c
    torch.cuda.empty_cache()
    return {"workload": f"{E} experts x {rows} tokens, N={N} K={K} MXFP4 per GPU",
            "ms_per_step": ms, "tflops_per_gpu": tf,
            "frac_of_measured": tf / tensor_peak("mxfp4", peaks),
            "launches_per_step": 2, "parity": parity}


def time_attention(world: int, peaks: dict, peak_src: str, steps: int, warmup: int) -> dict:
    """Attention forward leg: the reference FMHA bench's default problem
    (B=1, HQ=HK=64, S=8192, D=128, bf16, bhsd, non-causal) on every rank.
    q, k and v together are 384 MB, above the 126 MB L2."""
    from gfx950_gluon_tutorials_b200 import attention, ops
    B, H, S, D = 1, 64, 8192, 128
    dev = torch.device("cuda", torch.cuda.current_device())
    q, k, v, md = attention.input_helper(B, H, H, S, S, D, torch.bfloat16, "bhsd", device=dev)
    o = torch.empty_like(q)
    for _ in range(max(3, warmup)):
        attention.run_gluon_attention(q, k, v, o, md)
    barrier(world)
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        attention.run_gluon_attention(q, k, v, o, md)
    end.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(start.elapsed_time(end) / steps, world)
    ops.check_status()
    flops = attention.compute_flops(B, H, S, S, D, False)
    tf = flops / (ms * 1e-3) / 1e12
    # parity: 128 query rows of two heads against the float64 oracle under the
    # reference's tolerance rule (kernels/attention/common.py:142-174)
    from oracle import attention as oa
    import numpy as np
    checks = []
    for h, (r0, _) in zip((3, H - 5), pick_blocks(S, 128, 2, 733)):
        sl = slice(r0, r0 + 128)
        ref = oa.sdpa_tiles(q[:, h:h + 1].float().cpu().numpy(),
                            k[:, h:h + 1].float().cpu().numpy(),
                            v[:, h:h + 1].float().cpu().numpy(), md.sm_scale, sl)
        got = o[:, h:h + 1, sl].float().cpu().numpy()
        ok, dmax, _ = oa.check_output(got, ref, "bfloat16")
        checks.append((h, r0, ok, dmax, float(np.abs(ref).max())))
    parity = {"ok": all(x[2] for x in checks), "max_abs_diff": max(x[3] for x in checks),
              "rule": "reference _check_output: atol max(1e-3, 2 eps x max|ref|), rtol 1e-3",
              "blocks": [[h, r0] for h, r0, *_ in checks], "checker": "oracle (CPU, float64)"}
    del q, k, v, o
    torch.cuda.empty_cache()
    return {"workload": f"FMHA forward B={B} HQ=HK={H} S={S} D={D} bf16 bhsd non-causal per GPU",
            "ms_per_call": ms, "tflops_per_gpu": tf,
            "roofline": {"bound": "tensor", "achieved": tf, "peak": peaks["bf16_tflops"],
                         "unit": "TFLOP/s", "frac": tf / peaks["bf16_tflops"],
                         "algorithmic_flops_per_launch": flops,
                         "peak_source": f"{peak_src} bf16_tflops (burst)",
                         # the timed loop runs ~0.1 s under the power cap
                         "peak_sustained": peaks.get("bf16_tflops_sustained"),
                         "frac_of_sustained": (tf / peaks["bf16_tflops_sustained"]
                                               if peaks.get("bf16_tflops_sustained") else None)},
            "launches_per_call": 1, "parity": parity}


def time_allgather(w: Workload, world: int, iters: int = 10) -> dict | None:
    """Separately timed NCCL all-gather of every rank's C slab into a
    [world][M][N/world] buffer in each GPU's own memory."""
    if world == 1:
        return None
    from gfx950_gluon_tutorials_b200.shard import gather_slabs
    c = w.sets[0]["c"]
    for _ in range(3):
        out = gather_slabs(c)
    barrier(world)
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(iters):
        out = gather_slabs(c)
    end.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(start.elapsed_time(end) / iters, world)
    total = out.numel() * out.element_size()
    res = {"bytes": total, "ms": ms, "algbw_gbs": total / ms / 1e6,
           "busbw_gbs": total * (world - 1) / world / ms / 1e6}
    if w.dtype_name in ("fp16", "bf16"):
        res.update(time_gemm_gather(w, world, iters))
    return res


def time_gemm_gather(w: Workload, world: int, iters: int, chunks: int = 4) -> dict:
    """The slab GEMM followed by the gather of C, as one step: sequential
    (GEMM, then the NCCL all-gather) against `shard.gemm_gather_p2p` (row
    chunks written into a symmetric buffer, each chunk copied to the peers by
    the copy engines while the next chunk computes)."""
    from gfx950_gluon_tutorials_b200.shard import (P2P_MAX_WORLD, gather_slabs, gemm_gather,
                                                   gemm_gather_p2p)
    ops = w.ops
    s = w.sets[0]
    copy = torch.cuda.Stream()

    def sequential():
        return gather_slabs(ops.gemm_f16(s["a"], s["b"], s["c"]))

    def overlapped():
        return gemm_gather_p2p(lambda x, y, out: ops.gemm_f16(x, y, out), s["a"], s["b"],
                               chunks=chunks, out_dtype=s["c"].dtype, copy_stream=copy)

    def timed(fn):
        for _ in range(3):
            fn()
        barrier(world)
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(iters):
            fn()
        end.record()
        torch.cuda.synchronize()
        return max_over_ranks(start.elapsed_time(end) / iters, world)

    def chosen():
        return gemm_gather(lambda x, y, out: ops.gemm_f16(x, y, out), s["a"], s["b"],
                           chunks=chunks, out_dtype=s["c"].dtype, copy_stream=copy)

    seq = timed(sequential)
    ovl = timed(overlapped)
    auto = timed(chosen)
    ops.check_status()
    # parity of the peer copies: every slot of this rank's buffer equals the
    # NCCL all-gather of the slabs each rank computed into its own slot
    rank = torch.distributed.get_rank()
    buf = overlapped()
    torch.cuda.synchronize()
    ref = gather_slabs(buf[rank].contiguous())
    ok = torch.tensor([1 if torch.equal(ref, buf) else 0], device=buf.device)
    torch.distributed.all_reduce(ok, op=torch.distributed.ReduceOp.MIN)
    return {"gemm_then_gather_ms": seq, "gemm_gather_p2p_overlapped_ms": ovl,
            "gemm_gather_ms": auto,
            "gemm_gather_path": ("p2p overlap" if world <= P2P_MAX_WORLD
                                 else "GEMM then NCCL all-gather"),
            "overlap_chunks": chunks, "gather_parity_ok": bool(ok.item() == 1),
            "gather_parity_check": "p2p-gathered [world][M][n] buffer equals the NCCL "
                                   "all-gather of each rank's own slot (torch.equal)"}


LARGE_M, LARGE_N, LARGE_K = 16384, 53248, 16384


def _large_operands(dev, lo: int, hi: int, with_a: bool = True) -> dict:
    """BASELINE configs[4] operands: A (16384 x 16384) and B rows [lo, hi) of
    the 53248 x 16384 weight, N(0,1) quantised to MXFP4 by the config-3 rule.
    B is drawn in 256-row blocks from generators seeded by block index, so a
    shard is bit-identical to the same rows of the whole matrix at any GPU
    count. Scales are stored as the reference stores them (M-contiguous)."""
    from gfx950_gluon_tutorials_b200 import ops
    K = LARGE_K
    out = {}
    if with_a:
        g = torch.Generator(device=dev).manual_seed(4000)
        x = torch.randn((LARGE_M, K), generator=g, device=dev)
        out["a"], out["sa"] = ops.quantize_mxfp4(x, rows_pad=LARGE_M)
        del x
    x = torch.empty((hi - lo, K), device=dev)
    for r in range(lo, hi, 256):
        g = torch.Generator(device=dev).manual_seed(5000 + r // 256)
        x[r - lo:min(hi, r + 256) - lo].normal_(generator=g)
    out["b"], out["sb"] = ops.quantize_mxfp4(x, rows_pad=hi - lo)
    del x
    return out


def _time_large_once(inp: dict, c: torch.Tensor, steps: int, warmup: int) -> float:
    from gfx950_gluon_tutorials_b200 import a4w4, ops
    for _ in range(warmup):
        a4w4.matmul(inp["a"], inp["b"], inp["sa"], inp["sb"], c)
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        a4w4.matmul(inp["a"], inp["b"], inp["sa"], inp["sb"], c)
    end.record()
    torch.cuda.synchronize()
    ops.check_status()
    return start.elapsed_time(end) / steps


def time_large(world: int, rank: int, peaks: dict, steps: int, warmup: int) -> dict:
    """MXFP4 C = A B^T, M = 16384, N = 53248, K = 16384,
    B split along N over the ranks (whole 256-column tiles), A replicated, no
    collective in the timed loop. Reports the max-over-ranks time, the
    aggregate rate, the single-GPU time of the whole problem measured in the
    same run (rank 0 alone, after the sharded run), the resulting speed-up and
    efficiency, per-rank parity of two seeded 128 x 128 blocks against the
    oracle, and (N > 1) the separately timed NCCL all-gather of the C slabs."""
    from gfx950_gluon_tutorials_b200.shard import gather_slabs, shard_range
    dev = torch.device("cuda", torch.cuda.current_device())
    M, N, K = LARGE_M, LARGE_N, LARGE_K
    lo, hi = shard_range(N, world, rank, align=256)
    inp = _large_operands(dev, lo, hi)
    c = torch.empty((M, hi - lo), dtype=torch.bfloat16, device=dev)
    barrier(world)
    ms = max_over_ranks(_time_large_once(inp, c, steps, warmup), world)
    parity = parity_gemm("mxfp4", inp, c, pick_blocks(M, hi - lo, 2, 6000 + rank))
    flops = 2.0 * M * N * K
    res = {"workload": "a4w4 MXFP4 16384x53248x16384, B split along N over the ranks, "
                       "A replicated (BASELINE configs[4])",
           "M": M, "N_total": N, "K": K, "N_per_gpu": hi - lo,
           "steps": steps, "warmup": warmup, "ms": ms,
           "tflops": flops / (ms * 1e-3) / 1e12,
           "tflops_per_gpu": flops / world / (ms * 1e-3) / 1e12}
    res["frac_of_measured"] = res["tflops_per_gpu"] / tensor_peak("mxfp4", peaks)
    # every rank's parity, gathered
    flag = torch.tensor([1.0 if parity["ok"] else 0.0, parity["max_norm_err"],
                         parity["bit_exact_frac"]], dtype=torch.float64, device=dev)
    if world > 1:
        allp = [torch.empty_like(flag) for _ in range(world)]
        torch.distributed.all_gather(allp, flag)
    else:
        allp = [flag]
    allp = [p.tolist() for p in allp]
    res["parity"] = {"ok": all(p[0] == 1.0 for p in allp), "tol": TOL["mxfp4"],
                     "per_rank": [{"rank": r, "ok": p[0] == 1.0, "max_norm_err": p[1],
                                   "bit_exact_frac": p[2]} for r, p in enumerate(allp)],
                     "blocks_per_rank": 2, "checker": "oracle (CPU)"}
    if world > 1:
        # the separately timed NCCL all-gather of the C slabs, and a check that
        # every gathered slot holds its owner's slab (checksums of checksums)
        for _ in range(2):
            out = gather_slabs(c)
        barrier(world)
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        iters = 5
        start.record()
        for _ in range(iters):
            out = gather_slabs(c)
        end.record()
        torch.cuda.synchronize()
        gms = max_over_ranks(start.elapsed_time(end) / iters, world)
        mine = c.view(torch.int16).to(torch.int64).sum().reshape(1)
        sums = [torch.empty_like(mine) for _ in range(world)]
        torch.distributed.all_gather(sums, mine)
        slot = out.view(torch.int16).to(torch.int64).sum(dim=(1, 2))
        ok = torch.equal(slot, torch.cat(sums))
        okt = torch.tensor([1 if ok else 0], device=dev)
        torch.distributed.all_reduce(okt, op=torch.distributed.ReduceOp.MIN)
        total = out.numel() * out.element_size()
        res["allgather"] = {"bytes": total, "ms": gms, "algbw_gbs": total / gms / 1e6,
                            "busbw_gbs": total * (world - 1) / world / gms / 1e6,
                            "parity_ok": bool(okt.item() == 1),
                            "check": "per-slot int16 checksums equal the owners' checksums"}
        del out
    del inp, c
    torch.cuda.empty_cache()
    # single-GPU time of the whole problem, in the same run
    if world == 1:
        n1 = ms
    else:
        barrier(world)
        n1 = 0.0
        if rank == 0:
            full = _large_operands(dev, 0, N)
            cf = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
            n1 = _time_large_once(full, cf, steps, warmup)
            del full, cf
            torch.cuda.empty_cache()
        n1 = max_over_ranks(n1, world)
    res["single_gpu_ms"] = n1
    res["single_gpu_tflops"] = flops / (n1 * 1e-3) / 1e12
    res["speedup_vs_single_gpu"] = n1 / ms
    res["efficiency"] = n1 / (world * ms)
    return res


def cpu_reference_tflops(M: int, N: int, K: int, budget_s: float, threads: int) -> dict:
    """The reference's CPU path (torch.matmul in fp16 on the host cores,
    kernels/gemm/intra_wave/a16w16/bench.py:183) on the whole BASELINE
    configs[0] problem: one warm-up, then the median of three runs. Falls back
    to a row sample when one run would take longer than `budget_s` / 4."""
    from oracle import reference_cpu
    return reference_cpu.time_a16w16_full(M, N, K, threads=threads, runs=3,
                                          max_run_s=budget_s / 4)


def read_traffic(kernel_key: str):
    try:
        with open(TRAFFIC_PATH) as f:
            return json.load(f).get(kernel_key)
    except (OSError, ValueError):
        return None


# ---------------------------------------------------------------- contract --
def contract_main(args):
    # the reference arm times a CPU path: a single process needs no GPU
    rank, world, local = dist_setup(args.gpus, cuda=args.impl != "reference")
    if args.impl == "reference":
        return reference_main(args, rank, world)
    import gfx950_gluon_tutorials_b200 as pkg
    pkg.lib()  # the CUDA library must load; there is no fallback
    peaks, peak_src = load_peaks()
    M, K = 4096, 8192
    n_local = 4096
    clocks = ClockSampler(local)
    head_name = args.dtype
    # enough rotating sets that one pass over them exceeds the 126 MB L2
    w = Workload("head", M, n_local, K, head_name, sets=1, seed=1234 + rank)
    per_set = w.set_bytes()
    nsets = max(2, min(8, int(640e6 // per_set) + 1))
    w = Workload("head", M, n_local, K, head_name, sets=nsets, seed=1234 + rank)
    clocks.start()
    marks: list = []
    ms = time_device(w, args.steps, args.warmup, world, marks)
    clock_info = clocks.stop((marks[0], marks[1]))
    head_parity = w.check(seed=4242 + rank)
    flops_total = w.flops * world
    value = flops_total / (ms * 1e-3) / 1e12
    per_gpu = value / world
    peak = tensor_peak(head_name, peaks)
    by_dtype = {}
    if not args.no_extra:
        # config 1's second case: 3840 x 3840 x 8192 fp16 (225 tiles)
        cases = [("fp16_3840x3840x8192", 3840, 3840, 8192, "fp16", 55),
                 ("bf8", M, n_local, K, "bf8", 99), ("mxfp4", M, n_local, K, "mxfp4", 99)]
        for key, m_, n_, k_, dn, seed in cases:
            wx = Workload(key, m_, n_, k_, dn, sets=4, seed=seed + rank)
            msx = time_device(wx, args.steps, args.warmup, world)
            tf = wx.flops * world / (msx * 1e-3) / 1e12
            by_dtype[key] = {
                "ms_per_step": msx, "tflops": tf, "tflops_per_gpu": tf / world,
                "pct_of_nominal_dense_peak": 100.0 * tf / world / NOMINAL_DENSE_TFLOPS[dn],
                "frac_of_measured": tf / world / tensor_peak(dn, peaks),
                "launches_per_step": wx.launches_per_step,
                "parity": wx.check(seed=77 + len(key) + rank)}
            del wx
            torch.cuda.empty_cache()
    e2e_ms, h2d, d2h = time_e2e(w, max(3, args.steps // 5), min(args.warmup, 3), world)
    e2e_val = flops_total / (e2e_ms * 1e-3) / 1e12
    gather = time_allgather(w, world)
    del w
    torch.cuda.empty_cache()
    skinny = None if args.no_extra else time_skinny(world, peaks, peak_src)
    moe = None if args.no_extra else time_moe(world, peaks, args.steps, args.warmup)
    attn = None if args.no_extra else time_attention(world, peaks, peak_src, args.steps,
                                                     args.warmup)
    large = None if args.no_large else time_large(world, rank, peaks, args.large_steps,
                                                  args.large_warmup)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_reference_tflops(M, n_local, K, args.cpu_budget, os.cpu_count() or 1)
    if world > 1:
        barrier(world)
    if rank == 0:
        traffic = read_traffic(f"{head_name}_{M}x{n_local}x{K}")
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "TFLOPS",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": head_name,
            "data": "synthetic (seeded N(0,1) inputs, BASELINE recipes)",
            "config": {
                "workload": (f"a16w16 {head_name} C=A*B^T M=4096 K=8192, 4096 columns of C per "
                             "GPU, B sharded along N, A replicated (BASELINE configs[1])"),
                "M": M, "N_per_gpu": n_local, "K": K, "N_total": n_local * world,
                "parallelism": f"N-shard x{world}, no collective in the timed loop",
                "l2": f"rotating {nsets} input sets, {nsets * per_set / 1e6:.0f} MB > 126 MB L2",
            },
            "tflops_per_gpu": per_gpu,
            "pct_of_nominal_dense_peak": 100.0 * per_gpu / NOMINAL_DENSE_TFLOPS[head_name],
            "parity": head_parity,
            "by_dtype": by_dtype,
            "roofline": {
                "bound": "tensor", "achieved": per_gpu, "peak": peak, "unit": "TFLOP/s",
                "frac": per_gpu / peak, "traffic": traffic,
                "traffic_source": ("ncu dram__bytes_read.sum + dram__bytes_write.sum of one "
                                   "cold-input launch (profiles/traffic.json)"
                                   if traffic is not None else None),
                "peak_source": (f"{peak_src} bf16_tflops (burst) x dtype ratio"
                                if head_name not in ("fp16", "bf16")
                                else f"{peak_src} bf16_tflops (burst)"),
                "algorithmic_flops_per_launch": w_flops(M, n_local, K),
                "algorithmic_bytes_per_launch": algo_bytes(head_name, M, n_local, K),
            },
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_val, "unit": "TFLOPS", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
                    "path": ("public API (a16w16.matmul) on pinned host buffers; each step "
                             "uploads its inputs and downloads its C, overlapped with the "
                             "neighbouring steps' GEMMs on separate streams")},
            "gpu_launches": args.steps * (1 if head_name in ("fp16", "bf16") else 2),
            "clocks": clock_info,
        }
        if gather is not None:
            line["allgather"] = gather
        if skinny is not None:
            line["skinny"] = skinny
        if moe is not None:
            line["moe_grouped_mxfp4"] = moe
        if attn is not None:
            line["attention_fwd"] = attn
        if large is not None:
            line["large"] = large
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


def w_flops(M: int, N: int, K: int) -> float:
    return 2.0 * M * N * K


def algo_bytes(dtype_name: str, M: int, N: int, K: int) -> int:
    """A + B (+ scales) + C bytes of one launch."""
    eb = {"fp16": 2, "bf16": 2, "bf8": 1, "mxfp4": 0.5}[dtype_name]
    scales = (M + N) * (K // 32) if dtype_name in ("bf8", "mxfp4") else 0
    return int((M + N) * K * eb + scales + M * N * 2)


def reference_main(args, rank, world):
    """CPU reference arm: rank 0 times the reference path; other ranks exit.
    Each step is one whole BASELINE configs[0] problem (a row sample only if
    one problem would take longer than --ref-step-s)."""
    if rank != 0:
        if world > 1:
            torch.distributed.destroy_process_group()
        return
    M, K, n_local = 4096, 8192, 4096
    threads = os.cpu_count() or 1
    from oracle import reference_cpu
    info = reference_cpu.time_a16w16_full(M, n_local, K, threads=threads,
                                          runs=args.steps, warmup=args.warmup,
                                          max_run_s=args.ref_step_s)
    value = info["value"]
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOPS", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp16",
        "data": "synthetic (seeded N(0,1)/sqrt(K) inputs, BASELINE configs[0])",
        "impl": "reference",
        "config": {"workload": "a16w16 fp16 C=A*B^T M=4096 N=4096 K=8192 (BASELINE configs[0]/[1]) "
                               "on the host cores", "M": M, "N_per_gpu": n_local, "K": K},
        "ms_per_step": info["ms_per_run"],
        "cpu_baseline": {"value": value, "unit": "TFLOPS", "cores": info["cores"],
                         "kind": "port", "sample": info["sample"]},
        "e2e": {"value": value, "unit": "TFLOPS", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


# ------------------------------------------------- reference bench surface --
def surface_call(kernel: str, dn: str, M: int, N: int, K: int, seed: int,
                 prepared: bool = False):
    """A fresh input set of the reference bench's recipe and the call on it,
    C preallocated (the rotating copies of a, b and c). `prepared`: the call as
    an ops.PreparedGemm (the reference's --prepared route,
    scripts/benchmark_prepared.py), planned once and then only launched."""
    from gfx950_gluon_tutorials_b200 import a4w4, a8w8, a16w16, ops
    g = torch.Generator(device="cuda").manual_seed(1000 + seed)
    if kernel == "a16w16":
        dt = torch.float16 if dn == "fp16" else torch.bfloat16
        a = torch.randn((M, K), generator=g, device="cuda").to(dt)
        b = torch.randn((N, K), generator=g, device="cuda").to(dt).T
        c = torch.empty((M, N), device="cuda", dtype=dt)
        if prepared:
            return ops.prepare_gemm_f16(a, b.T, c)
        return lambda: a16w16.matmul(a, b, c)
    if kernel == "a8w8":
        a = (torch.rand((M, K), generator=g, device="cuda").half() - 0.5).to(torch.float8_e5m2)
        b = (torch.rand((N, K), generator=g, device="cuda").half().T - 0.5).to(torch.float8_e5m2)
        if prepared:
            return ops.prepare_gemm_f8(a, b.T, torch.empty((M, N), device="cuda",
                                                           dtype=torch.float16))
        return lambda: a8w8.matmul(a, b)
    a = torch.randint(0, 256, (M, K // 2), generator=g, device="cuda", dtype=torch.uint8)
    b = torch.randint(0, 256, (N, K // 2), generator=g, device="cuda", dtype=torch.uint8)
    m_pad = (M + 255) // 256 * 256
    sa = torch.randint(124, 128, (K // 32, m_pad), generator=g, device="cuda",
                       dtype=torch.uint8).T[:M]
    sb = torch.randint(124, 128, (K // 32, N), generator=g, device="cuda", dtype=torch.uint8).T
    c = torch.empty((M, N), device="cuda", dtype=torch.bfloat16)
    if prepared:
        return ops.prepare_gemm_mxf4(a, b, sa, sb, c)
    return lambda: a4w4.matmul(a, b, sa, sb, c)


def reference_surface_main(args):
    """kernels/gemm/intra_wave/<kind>/bench.py: correctness then a TFLOPS table."""
    from gfx950_gluon_tutorials_b200 import a4w4, a8w8, a16w16, ops
    torch.cuda.set_device(0)
    if args.version is not None:
        print(f"[{args.kernel}] --version {args.version}: this build has one kernel per kind "
              f"(gemm_kernel, tcgen05); running it", flush=True)
    ks = [args.K] if args.K else [512, 1024, 2048, 4096, 8192, 16384, 32768]
    M, N = args.M, args.N
    dtypes = args.dtype or (["fp16", "bf16"] if args.kernel == "a16w16" else ["-"])
    rows = []
    for dn in dtypes:
        for K in ks:
            if args.kernel == "a16w16":
                dt = torch.float16 if dn == "fp16" else torch.bfloat16
                a = torch.rand((M, K), device="cuda", dtype=dt) - 0.5
                b = torch.rand((N, K), device="cuda", dtype=dt).T - 0.5
                ok = torch.allclose(a16w16.matmul(a, b), torch.matmul(a, b), atol=1e-1, rtol=0)
                fn = lambda: a16w16.matmul(a, b)  # noqa: E731
                elem = a.element_size()
            elif args.kernel == "a8w8":
                a = (torch.rand((M, K), device="cuda", dtype=torch.float16) - 0.5).to(
                    torch.float8_e5m2)
                b = (torch.rand((N, K), device="cuda", dtype=torch.float16).T - 0.5).to(
                    torch.float8_e5m2)
                ref = torch.matmul(a.to(torch.float16), b.to(torch.float16))
                ok = torch.allclose(a8w8.matmul(a, b), ref, atol=1e-1, rtol=0)
                fn = lambda: a8w8.matmul(a, b)  # noqa: E731
                elem = 1
            else:
                gen = torch.Generator().manual_seed(42)
                a = ((torch.randint(0, 16, (M, K // 2), generator=gen, dtype=torch.uint8) << 4)
                     | torch.randint(0, 16, (M, K // 2), generator=gen, dtype=torch.uint8)).cuda()
                b = ((torch.randint(0, 16, (N, K // 2), generator=gen, dtype=torch.uint8) << 4)
                     | torch.randint(0, 16, (N, K // 2), generator=gen, dtype=torch.uint8)).cuda()
                m_pad = (M + 255) // 256 * 256
                sa = torch.randint(124, 128, (K // 32, m_pad), dtype=torch.uint8).cuda().T[:M]
                sb = torch.randint(124, 128, (K // 32, N), dtype=torch.uint8).cuda().T
                from oracle import mx
                ref = mx.bf16_bits_to_f32(mx.gemm_mxfp4_ref(a.cpu().numpy(), b.cpu().numpy(),
                                                            sa.cpu().numpy(), sb.cpu().numpy()))
                got = a4w4.matmul(a, b, sa, sb).float().cpu().numpy()
                ok = bool(abs(got - ref).max() <= 0.1)
                fn = lambda: a4w4.matmul(a, b, sa, sb)  # noqa: E731
                elem = 0.5
            ops.check_status()
            print(f"[{args.kernel}] M={M} N={N} K={K} dtype={dn}: "
                  f"{'match' if ok else 'DIFFER'}", flush=True)
            if args.rocprof:
                # cold caches as kernels/gemm/intra_wave/a16w16/bench.py:190-241
                # does it: enough copies of (a, b, c) to fill --rotating-buffer-size
                # MB, launch i using copy i % copies
                set_bytes = int((M + N) * K * elem) + M * N * 2
                copies = max(1, args.rotating_buffer_size * 1024 * 1024 // set_bytes)
                calls = [surface_call(args.kernel, dn, M, N, K, i, args.prepared)
                         for i in range(copies)]
                print(f"[{args.kernel}] M={M} N={N} K={K} dtype={dn}: rotating tensors: "
                      f"{copies} copies, {copies * set_bytes / 1024 ** 2:.0f} MB", flush=True)
                calls[0]()
                torch.cuda.synchronize()
                for i in range(1000):
                    calls[i % copies]()
                torch.cuda.synchronize()
                ops.check_status()
                del calls
                print(f"[{args.kernel}] M={M} N={N} K={K}: 1000 iterations done", flush=True)
                continue
            if args.prepared:
                fn = surface_call(args.kernel, dn, M, N, K, 0, prepared=True)
            for _ in range(5):
                fn()
            st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            st.record()
            for _ in range(50):
                fn()
            en.record()
            torch.cuda.synchronize()
            ms = st.elapsed_time(en) / 50
            rows.append((M, N, K, dn, 2 * M * N * K / ms / 1e9, (M + N) * K * elem))
    if rows:
        print(f"{'M':>6} {'N':>6} {'K':>6} {'dtype':>6} {'TFLOPS':>9}")
        for M_, N_, K_, dn, tf, _ in rows:
            print(f"{M_:>6} {N_:>6} {K_:>6} {dn:>6} {tf:>9.1f}")


def main():
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b2g", "reference"], default="b2g")
    ap.add_argument("--config", choices=["default", "large"], default="default",
                    help="large: only the headline and the BASELINE configs[4] object")
    ap.add_argument("--dtype", nargs="+", default=None)
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the 3840^2/BF8/MXFP4, small-M, MoE and attention entries")
    ap.add_argument("--no-large", action="store_true",
                    help="skip the BASELINE configs[4] (16384x53248x16384 MXFP4) object")
    ap.add_argument("--large-steps", type=int, default=2,
                    help="timed launches of configs[4] (about 7.5 s each on one GPU)")
    ap.add_argument("--large-warmup", type=int, default=1)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--cpu-budget", type=float, default=8.0, help="seconds of CPU baseline work")
    ap.add_argument("--ref-step-s", type=float, default=4.0,
                    help="seconds of CPU work per --impl reference step")
    # reference bench surface
    ap.add_argument("--kernel", choices=["a16w16", "a8w8", "a4w4"], default=None)
    ap.add_argument("--version", type=int, default=None,
                    help="the reference's tutorial version; this build has one kernel per "
                         "kind, which every version runs (the surface says so)")
    ap.add_argument("--K", type=int, default=None)
    ap.add_argument("--M", type=int, default=4096)
    ap.add_argument("--N", type=int, default=4096)
    ap.add_argument("--rocprof", "--profile", dest="rocprof", action="store_true")
    ap.add_argument("--prepared", action="store_true",
                    help="time (or, with --rocprof, launch) prepared calls: planned once, "
                         "then only launched (the reference's --prepared route)")
    ap.add_argument("--rotating-buffer-size", type=int, default=512)
    args = ap.parse_args()
    if args.kernel is not None:
        return reference_surface_main(args)
    if args.dtype is None:
        args.dtype = "fp16"
    elif isinstance(args.dtype, list):
        args.dtype = args.dtype[0]
    if args.warmup < 3:
        log("note: raising --warmup to 3 (timing rule)")
        args.warmup = 3
    if args.config == "large":
        args.no_extra = True
        args.no_large = False
    contract_main(args)


if __name__ == "__main__":
    main()
