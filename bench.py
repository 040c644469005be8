"""Offline serving throughput: output tokens / s of ``LLM.generate`` on the headline workload
(the reference's offline benchmark, benchmark/offline/bench.py).

Model: Qwen3-14B architecture (bf16, random N(0, 0.02) weights), TP = number of GPUs.
Workload: 256 requests, prompt lengths U[100, 1024] with uniform random token ids, output lengths
U[100, 1024], greedy, EOS ignored. One *step* = one ``generate`` over the whole workload.

``python bench.py --gpus N --steps K --warmup W [--impl ours|reference] [--model qwen3-14b]``
For N > 1 run under ``torchrun --nproc-per-node N``; rank 0 prints one JSON line. The reference arm
(``--impl reference``) runs the unmodified reference installed in ``baseline/_ref``: its ``LLM`` at
N = 1 and, per torchrun rank, its own offline-mode ``Scheduler`` at N > 1.
"""

from __future__ import annotations

import argparse
import json
import os
import random
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))

# gpt-oss-120b (MoE): its experts stay MXFP4 in HBM (~65 GB of weights in all, so one GPU holds it);
# with MINISGL_MXFP4_RESIDENT=0 they are bf16 (~240 GB: TP >= 2); with MINISGL_MOE_PARALLEL=ep each
# rank holds whole experts
MODELS = {"qwen3-14b": "qwen3-14b", "qwen3-0.6b": "qwen3-0.6b", "qwen3-32b": "qwen3-32b",
          "gpt-oss-120b": "gpt-oss-120b"}
CONFIG = dict(max_running_req=256, cuda_graph_max_bs=256, page_size=64, max_seq_len_override=4096,
              max_extend_tokens=16384)


def workload(n: int, seed: int = 0, vocab: int = 151936):
    rng = random.Random(seed)
    prompts = [[rng.randint(0, vocab - 1) for _ in range(rng.randint(100, 1024))] for _ in range(n)]
    outs = [rng.randint(100, 1024) for _ in range(n)]
    return prompts, outs


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.idx = device_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for n, v in zip(names, parts[3:7]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def model_dir(preset: str, rank: int) -> str:
    sys.path.insert(0, ROOT)
    from minisgl.models.synthetic import make_checkpoint

    path = os.path.join(tempfile.gettempdir(), f"minisgl_bench_{preset}_{rank}")
    make_checkpoint(preset, path, weights=False)
    return path


def run(args, impl: str):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    preset = MODELS[args.model]
    path = model_dir(preset, rank)  # before the reference's package shadows ours
    prompts, outs = workload(args.num_reqs, args.seed)
    total_out = sum(outs)

    if impl == "reference":
        ref_root = os.path.join(ROOT, "baseline", "_ref")
        if not os.path.isdir(os.path.join(ref_root, "minisgl")):
            print(json.dumps({"impl": "reference", "unavailable":
                              "the reference is not installed in baseline/_ref (pip install --target baseline/_ref)"}))
            return
        sys.path[:] = [p for p in sys.path if os.path.abspath(p or ".") != ROOT]
        sys.path.insert(0, ref_root)
        for m in [m for m in sys.modules if m == "minisgl" or m.startswith("minisgl.")]:
            del sys.modules[m]
        os.chdir(tempfile.gettempdir())
        from minisgl.core import SamplingParams
        from minisgl.llm import LLM

        assert "baseline" in (getattr(sys.modules["minisgl.llm"], "__file__", "") or ""), "reference not isolated"
        if world == 1:
            llm = LLM(path, dtype=torch.bfloat16, use_dummy_weight=True, **CONFIG)
        else:
            # The reference's LLM constructor fixes tp_info to (0, 1) (python/minisgl/llm/llm.py:
            # 29-36); everything else about offline mode works per rank (its scheduler I/O picks the
            # offline receive/send methods for every rank, python/minisgl/scheduler/io.py:30-33).
            # So each torchrun rank builds the reference's own Scheduler with its rank's tp_info and
            # runs the stock LLM.generate loop; the engine, pynccl, cuBLAS and FlashInfer paths are
            # the reference's, unmodified.
            from minisgl.distributed import DistributedInfo
            from minisgl.scheduler import Scheduler, SchedulerConfig

            # the reference's engine rendezvouses on its own tcp://127.0.0.1:2333 store, hosted by
            # rank 0; under torchrun that variable would make every rank a client of the agent's
            # store instead, and nobody would host 2333
            os.environ.pop("TORCHELASTIC_USE_AGENT_STORE", None)

            class RankLLM(LLM):
                def __init__(self, model_path, dtype, **kwargs):
                    Scheduler.__init__(self, SchedulerConfig(model_path=model_path, dtype=dtype, offline_mode=True,
                                                             tp_info=DistributedInfo(rank, world), **kwargs))
                    self.pending_requests, self.status_map, self.counter = [], {}, 0  # its LLM.__init__ state

            llm = RankLLM(path, torch.bfloat16, use_dummy_weight=True, **CONFIG)
        with torch.no_grad():  # the reference's dummy init is N(0, 1); rescale to N(0, 0.02)
            for k, v in llm.engine.model.state_dict().items():
                if v.is_floating_point() and "norm" not in k:
                    v.mul_(0.02)
        dev = torch.device(f"cuda:{local}")
        cpu_group = llm.tp_cpu_group if world > 1 else None
    else:
        sys.path.insert(0, ROOT)
        from minisgl.core import SamplingParams
        from minisgl.llm import LLM

        llm = LLM(path, dtype=torch.bfloat16, use_dummy_weight=True, **CONFIG)
        dev = llm.engine.device
        cpu_group = llm.engine.tp_cpu_group

    sps = [SamplingParams(temperature=0.0, ignore_eos=True, max_tokens=o) for o in outs]

    def step():
        res = llm.generate(prompts, sps)
        n = sum(len(r["token_ids"]) for r in res)
        if n != total_out:
            raise RuntimeError(f"generated {n} tokens, expected {total_out}")

    for _ in range(args.warmup):
        step()

    counters = getattr(llm.engine, "counters", None)
    if counters is not None:
        counters.reset()
    sampler = ClockSampler(torch.cuda.current_device())
    if world > 1:
        dist.barrier(group=cpu_group)
    torch.cuda.synchronize(dev)
    sampler.start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    end.record()
    torch.cuda.synchronize(dev)
    wall = time.perf_counter() - t0
    if world > 1:
        dist.barrier(group=cpu_group)
    clocks = sampler.stop()
    dev_ms = start.elapsed_time(end) / args.steps
    wall_ms = wall * 1000 / args.steps
    if world > 1:
        t = torch.tensor([dev_ms, wall_ms], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=cpu_group)
        dev_ms, wall_ms = float(t[0]), float(t[1])
    if rank != 0:
        close(llm, impl, world)
        return
    line = {
        "metric": "offline output tok/s Qwen3-14B @TP1/2/4/8 B200" if args.model == "qwen3-14b"
        else f"offline output tok/s {args.model}",
        "value": round(total_out / (dev_ms / 1000), 2),
        "unit": "tok/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(dev_ms, 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (random token ids; random-init N(0,0.02) weights)",
        "config": {"model": args.model, "global_batch": args.num_reqs, "seq_len": "in U[100,1024], out U[100,1024]",
                   "parallelism": f"tp{args.gpus}", "output_tokens_per_step": total_out,
                   "l2": "inputs larger than L2 (weights + KV cache >> 126 MB)", **CONFIG},
        "clocks": clocks,
    }
    if impl == "reference":
        line["impl"] = "reference"
    if counters is not None:
        c = counters.snapshot()
        line["e2e"] = {"value": round(total_out / (wall_ms / 1000), 2), "unit": "tok/s",
                       "h2d_bytes_per_step": c["h2d_bytes"] // args.steps,
                       "d2h_bytes_per_step": c["d2h_bytes"] // args.steps}
        line["gpu_launches"] = c["launches"]
    else:
        line["e2e"] = {"value": round(total_out / (wall_ms / 1000), 2), "unit": "tok/s",
                       "h2d_bytes_per_step": None, "d2h_bytes_per_step": None}
    print(json.dumps(line), flush=True)
    close(llm, impl, world)


def close(llm, impl: str, world: int) -> None:
    if impl != "reference":
        llm.shutdown()
    elif world > 1:
        # CUDA graphs that hold NCCL calls go before the process group (the reference's own order)
        llm.engine.shutdown()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--model", choices=sorted(MODELS), default="qwen3-14b")
    ap.add_argument("--num-reqs", type=int, default=256)
    ap.add_argument("--seed", type=int, default=0)
    args = ap.parse_args()
    run(args, args.impl)


if __name__ == "__main__":
    main()
