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


class ClockSampler:
    """``nvidia-smi`` samples of the SM clock and the throttle reasons of one GPU every 200 ms
    between ``start()`` and ``stop()`` (a benchmark's timed region); ``stop()`` returns the median SM
    clock under load, the maximum clock and every throttle reason that was active."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, device_index: int):
        self.idx = device_index
        self.proc = None
        self.path = None

    def start(self) -> None:
        import os
        import subprocess
        import tempfile

        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        import os
        import statistics

        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait()
        sm, mx, reasons = [], [], set()
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for n, v in zip(self.REASONS, parts[3:7]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}
