"""Kernel timing helpers (reference: python/minisgl/benchmark/perf.py:10-74): CUDA-graph
amplified event timing, and bandwidth comparison against a baseline callable."""

from __future__ import annotations

from typing import Callable

import torch


def perf_cuda(fn: Callable[[], object], *, warmup: int = 3, reps: int = 20, graph_calls: int = 10) -> float:
    """Mean milliseconds per call of ``fn``: ``graph_calls`` calls captured in one CUDA graph,
    replayed ``reps`` times, timed with CUDA events on the capturing stream."""
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for _ in range(warmup):
            fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for _ in range(graph_calls):
            fn()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(s):  # replays and both events on one stream
        g.replay()
        torch.cuda.synchronize()
        a.record(s)
        for _ in range(reps):
            g.replay()
        b.record(s)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / (reps * graph_calls)


def compare_memory_kernel_perf(ours: Callable[[], object], baseline: Callable[[], object], nbytes: int,
                               name: str = "kernel") -> dict:
    t0, t1 = perf_cuda(ours), perf_cuda(baseline)
    res = {"name": name, "ours_ms": t0, "baseline_ms": t1, "ours_gbs": nbytes / t0 / 1e6,
           "baseline_gbs": nbytes / t1 / 1e6, "speedup": t1 / t0}
    print(f"{name}: ours {res['ours_gbs']:.0f} GB/s, baseline {res['baseline_gbs']:.0f} GB/s, x{res['speedup']:.2f}")
    return res
