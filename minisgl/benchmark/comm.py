"""Tensor-parallel collective micro-benchmark, one process per GPU:

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m minisgl.benchmark.comm [--hidden 5120]

For each token count it times, on decode-sized activations [T, hidden] bf16:

* ``nvls``  - the fused NVLS all-reduce + residual add + RMSNorm kernel (one launch);
* ``peer``  - the IPC peer-memory all-reduce followed by the fused add + RMSNorm kernel;
* ``nccl``  - NCCL all-reduce (torch.distributed) followed by the same norm kernel (the baseline);
* ``gemm_nvls`` - the row-parallel GEMM ``[T, K] x [hidden, K]^T`` (``--k``, default the Qwen3-14B
  o_proj shard 5120 / N) fused with the collective: the GEMM writes the NVLS staging region and
  signals arrival, then reduce-scatter + residual + RMSNorm + all-gather (the engine's decode path);
* ``gemm_nccl`` - the same GEMM, then NCCL all-reduce and the norm kernel (the reference's shape of
  the step: cuBLAS GEMM, NCCL all-reduce, fused_add_rmsnorm).

Each variant runs 20 times inside one CUDA graph, replayed 10 times; the CUDA-event time per call
is the MAX over ranks. Rooflines: for the collective alone, the slower of the bytes each GPU must
move over NVLink (reduce-scatter in + all-gather out: 2 x T x hidden x 2 x (N-1)/N) at the measured
770 GB/s per direction and the norm's HBM traffic at the measured copy bandwidth; for the GEMM
variants, the slower of that and the GEMM's own bound (FLOPs at the measured bf16 peak, weight bytes
at HBM bandwidth). Rank 0 prints one JSON line per token count with each variant's time and its
fraction of its roofline.
"""

from __future__ import annotations

import argparse
import json
import os
from datetime import timedelta

import torch
import torch.distributed as dist

NVLINK_BPS = 770e9  # measured peer copy, per direction per GPU


def _peaks() -> tuple:
    """(HBM bytes/s, bf16 FLOP/s burst) measured on this pool, or the fallback figures."""
    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    try:
        with open(os.path.join(root, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]) * 1e9, float(d["bf16_tflops"]) * 1e12
    except (OSError, KeyError, ValueError):
        return 6.65e12, 1.59e15


def _time(fn, stream, calls: int = 20, reps: int = 10) -> float:
    """Milliseconds per call: ``calls`` calls captured in one graph, replayed ``reps`` times."""
    with torch.cuda.stream(stream):
        for _ in range(3):
            fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for _ in range(calls):
            fn()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        g.replay()
        torch.cuda.synchronize()
        a.record(stream)
        for _ in range(reps):
            g.replay()
        b.record(stream)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / (calls * reps)
    del g
    return ms


def _trace(nvls, x, xin, wt, res, w, eps, rank: int, T: int) -> None:
    """Phase spans (us) of one RS call, from the kernel's %globaltimer stamps: start (after the
    producer wait) -> staged/arrived -> first barrier passed -> rows reduced, normalised and
    gathered -> second arrival -> second barrier (CTA 0). Medians over the CTAs that own rows."""
    import statistics

    tr = torch.zeros(128 * 8, dtype=torch.int64, device=x.device)
    out = {}
    for name in ("stage", "gemm"):
        for _ in range(3):
            if name == "gemm":
                y = nvls.linear_into_staging(xin, wt, None)
                nvls.all_reduce_add_rmsnorm(y, res, w, eps, trace=tr)
            else:
                nvls.all_reduce_add_rmsnorm(x, res, w, eps, trace=tr)
        torch.cuda.synchronize()
        grid = min(128, -(-(-(-T // nvls.world)) // 2))  # the RS launch: two rows in flight per CTA
        t = tr.view(128, 8)[:grid].cpu()
        t0 = int(t[:, 0].min())
        active = list(range(grid))
        span = lambda i, j: statistics.median(float(t[b, j] - t[b, i]) / 1e3 for b in active)
        out[name] = {"start_spread": round(float(t[:, 0].max() - t0) / 1e3, 2), "arrive1": round(span(0, 1), 2),
                     "wait1": round(span(1, 2), 2), "rows": round(span(2, 3), 2), "arrive2": round(span(3, 4), 2),
                     "wait2_cta0": round(float(t[0, 5] - t[0, 4]) / 1e3, 2),
                     "total_cta0": round(float(t[0, 5] - t0) / 1e3, 2)}
    if rank == 0:
        print(json.dumps({"trace_tokens": T, **out}), flush=True)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser("minisgl.benchmark.comm")
    ap.add_argument("--hidden", type=int, default=5120)
    ap.add_argument("--tokens", default="1,8,16,64,128,256,512")
    ap.add_argument("--k", type=int, default=0, help="GEMM input features per rank (0: 5120 / N)")
    ap.add_argument("--trace", action="store_true",
                    help="also print per-phase %%globaltimer spans of the reduce-scatter form (rank 0)")
    a = ap.parse_args(argv)
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    cpu = dist.new_group(backend="gloo", timeout=timedelta(seconds=60))
    from minisgl import ops
    from minisgl.parallel.comm import TorchDistributedImpl
    from minisgl.parallel.nvls import NvlsNormComm
    from minisgl.parallel.peer import PeerCommImpl

    H, eps = a.hidden, 1e-6
    tokens = [int(t) for t in a.tokens.split(",")]
    cap = max(tokens) * H * 2
    nccl = TorchDistributedImpl()
    peer = PeerCommImpl(cpu, dev, cap, nccl)
    try:
        nvls = NvlsNormComm(dist.group.WORLD, cpu, dev, cap)
    except RuntimeError as e:
        nvls = None
        if rank == 0:
            print(json.dumps({"nvls": f"unavailable: {e}"}), flush=True)
    s = torch.cuda.Stream()
    from .perf import ClockSampler

    clocks = ClockSampler(local)
    clocks.start()
    w = (torch.rand(H, device=dev) + 0.5).to(torch.bfloat16)
    hbm, flops = _peaks()
    K = a.k or 5120 // world
    wt = (torch.randn(H, K, device=dev) * 0.02).to(torch.bfloat16)
    for T in tokens:
        x = torch.randn(T, H, device=dev, dtype=torch.bfloat16)
        res = torch.randn(T, H, device=dev, dtype=torch.bfloat16)
        times = {}
        if nvls is not None:
            times["nvls"] = _time(lambda: nvls.all_reduce_add_rmsnorm(x, res, w, eps), s)

        ybuf = x.clone()

        def unfused(impl):
            # NCCL reduces in place and the norm then overwrites the sum with normalised rows, so
            # repeated calls stay bounded; the peer all-reduce returns a new tensor
            def run():
                y = impl.all_reduce(ybuf)
                ops.fused_add_rmsnorm(y, res, w, eps)
            return run

        times["peer"] = _time(unfused(peer), s)
        times["nccl"] = _time(unfused(nccl), s)
        xin = (torch.randn(T, K, device=dev) * 0.5).to(torch.bfloat16)
        if nvls is not None:
            def gemm_nvls():
                y = nvls.linear_into_staging(xin, wt, None)
                if y is None:  # LL-sized batch: plain GEMM, then the LL collective
                    y = ops.linear(xin, wt)
                nvls.all_reduce_add_rmsnorm(y, res, w, eps)

            times["gemm_nvls"] = _time(gemm_nvls, s)

        def gemm_nccl():
            y = nccl.all_reduce(ops.linear(xin, wt))
            ops.fused_add_rmsnorm(y, res, w, eps)

        times["gemm_nccl"] = _time(gemm_nccl, s)
        t = torch.tensor([times[k] for k in sorted(times)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=cpu)
        times = {k: float(v) for k, v in zip(sorted(times), t)}
        nbytes = T * H * 2
        link = 2 * nbytes * (world - 1) / world  # reduce-scatter in + all-gather out, per GPU
        roof_ms = max(link / NVLINK_BPS, 4 * nbytes / hbm) * 1e3  # norm: x, residual in/out, out
        gemm_ms = max(2 * T * K * H / flops, K * H * 2 / hbm) * 1e3
        if rank == 0:
            row = {"world": world, "tokens": T, "hidden": H, "k": K, "roofline_us": round(roof_ms * 1e3, 2),
                   "gemm_roofline_us": round(max(roof_ms, gemm_ms) * 1e3, 2)}
            for k, v in times.items():
                r = max(roof_ms, gemm_ms) if k.startswith("gemm") else roof_ms
                row[f"{k}_us"] = round(v * 1e3, 2)
                row[f"{k}_frac"] = round(r / v, 3)
            print(json.dumps(row), flush=True)
        if a.trace and nvls is not None and not nvls.is_ll(T, H):
            _trace(nvls, x, xin, wt, res, w, eps, rank, T)
    torch.cuda.synchronize()
    c = clocks.stop()
    clk = [None] * world
    dist.all_gather_object(clk, c, group=cpu)
    if rank == 0:
        print(json.dumps({"clocks": clk}), flush=True)
    dist.barrier(group=cpu)
    if nvls is not None:
        nvls.close()
    peer.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
