"""The reference's CPU path, timed - TEST / BASELINE INFRASTRUCTURE ONLY.

The reference checks every GEMM against torch on the same inputs
(kernels/gemm/intra_wave/a16w16/bench.py:183: ``torch.matmul(a, b)`` in the
input dtype). Run on the host cores, that expression is the CPU baseline the
B200 kernels are reported next to. Only bench.py's CPU-baseline leg and its
``--impl reference`` arm call this module.
"""

from __future__ import annotations

import time

import torch


def time_a16w16(M: int, N: int, K: int, budget_s: float = 8.0, threads: int = 1,
                sample_rows: int = 512, seed: int = 0) -> dict:
    """TFLOP/s of torch.matmul(a, b) in fp16 on the CPU for a row sample of the
    M x N x K workload (inputs N(0,1)/sqrt(K) like BASELINE configs[0]),
    repeated until about ``budget_s`` seconds have been spent."""
    torch.set_num_threads(max(1, threads))
    g = torch.Generator().manual_seed(seed)
    rows = min(M, sample_rows)
    a = (torch.randn((rows, K), generator=g) / K ** 0.5).half()
    b = (torch.randn((N, K), generator=g) / K ** 0.5).half().T   # (K, N) view, as the bench
    torch.matmul(a[:8], b)  # warm the kernels / thread pool
    reps, spent = 0, 0.0
    t_end = time.perf_counter() + budget_s
    while True:
        t0 = time.perf_counter()
        torch.matmul(a, b)
        spent += time.perf_counter() - t0
        reps += 1
        if time.perf_counter() >= t_end:
            break
    flops = 2.0 * rows * N * K * reps
    return {
        "value": flops / spent / 1e12,
        "unit": "TFLOPS",
        "cores": torch.get_num_threads(),
        "kind": "port",
        "sample": (f"torch.matmul fp16 on CPU, {rows} of {M} rows x N={N} x K={K}, "
                   f"{reps} reps in {spent:.1f} s"),
    }


def time_a16w16_full(M: int, N: int, K: int, threads: int = 1, runs: int = 3,
                     warmup: int = 1, max_run_s: float = 4.0, seed: int = 0) -> dict:
    """TFLOP/s of torch.matmul(a, b) in fp16 on the CPU for the whole M x N x K
    problem (inputs N(0,1)/sqrt(K)): `warmup` untimed
    runs, then the median of `runs` timed ones. If the first run takes longer
    than `max_run_s`, the timed runs use the largest row sample that fits it
    instead, and the sample says so."""
    import statistics
    torch.set_num_threads(max(1, threads))
    g = torch.Generator().manual_seed(seed)
    a = (torch.randn((M, K), generator=g) / K ** 0.5).half()
    b = (torch.randn((N, K), generator=g) / K ** 0.5).half().T   # (K, N) view, as the bench
    t0 = time.perf_counter()
    torch.matmul(a, b)
    first = time.perf_counter() - t0
    rows = M
    if first > max_run_s:
        rows = max(8, int(M * max_run_s / first) // 8 * 8)
        a = a[:rows]
    for _ in range(max(0, warmup - 1)):
        torch.matmul(a, b)
    times = []
    for _ in range(max(1, runs)):
        t0 = time.perf_counter()
        torch.matmul(a, b)
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    what = "whole problem" if rows == M else f"{rows} of {M} rows (one run exceeded {max_run_s} s)"
    return {
        "value": 2.0 * rows * N * K / med / 1e12,
        "unit": "TFLOPS",
        "cores": torch.get_num_threads(),
        "kind": "port",
        "ms_per_run": med * 1e3 * M / rows,
        "sample": (f"torch.matmul fp16 on CPU, M={M} N={N} K={K} ({what}), "
                   f"{warmup} warm-up + median of {len(times)} runs"),
    }
