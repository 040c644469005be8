"""Tensor parallelism on CPU: two gloo ranks (one process each, launched like torchrun) must
produce exactly the TP1 greedy tokens of the fp32 oracle."""

import json
import os
import subprocess
import sys

import pytest
import torch

from minisgl.core import SamplingParams
from minisgl.models.synthetic import make_checkpoint

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

WORKER = r"""
import json, os, sys
sys.path.insert(0, {root!r})
import torch
from minisgl.core import SamplingParams
from minisgl.llm import LLM
prompts = json.loads(os.environ["TP_PROMPTS"])
llm = LLM({path!r}, dtype=torch.float32, device="cpu", max_running_req=16, cache_type="radix",
          max_extend_tokens=48)
out = [o["token_ids"] for o in llm.generate(prompts, SamplingParams(max_tokens=12, ignore_eos=True))]
llm.cache_manager.check_integrity()
if int(os.environ["RANK"]) == 0:
    print("RESULT " + json.dumps(out), flush=True)
llm.shutdown()
"""


def _prompts():
    g = torch.Generator().manual_seed(3)
    return [torch.randint(0, 1000, (int(torch.randint(8, 40, (1,), generator=g)),), generator=g).tolist()
            for _ in range(6)]


@pytest.mark.parametrize("preset,moe_parallel", [("tiny-qwen3", "tp"), ("tiny-qwen3-odd", "tp"), ("tiny-qwen3-moe", "tp"),
                                                  ("tiny-qwen3-moe", "ep"), ("tiny-gpt-oss", "tp"),
                                                  ("tiny-gpt-oss", "ep")])
def test_tp2_matches_tp1(tmp_path, preset, moe_parallel, free_port):
    """TP2 (experts sliced, or whole experts per rank with MINISGL_MOE_PARALLEL=ep) gives the TP1
    tokens; gpt-oss loads from its fused-expert checkpoint layout."""
    from minisgl.llm import LLM

    fmt = "fused" if preset == "tiny-gpt-oss" else "per_expert"
    path = make_checkpoint(preset, str(tmp_path / preset), expert_format=fmt)
    prompts = _prompts()
    llm = LLM(path, dtype=torch.float32, device="cpu", max_running_req=16, distributed_port=free_port,
              max_extend_tokens=48)
    try:
        ref = [o["token_ids"] for o in llm.generate(prompts, SamplingParams(max_tokens=12, ignore_eos=True))]
    finally:
        llm.shutdown()
    script = tmp_path / "worker.py"
    script.write_text(WORKER.format(root=ROOT, path=path))
    procs = []
    for r in range(2):
        env = dict(os.environ, RANK=str(r), LOCAL_RANK=str(r), WORLD_SIZE="2", MASTER_ADDR="127.0.0.1",
                   MASTER_PORT=str(free_port + 7), TP_PROMPTS=json.dumps(prompts), PYTHONPATH=ROOT,
                   MINISGL_MOE_PARALLEL=moe_parallel)
        procs.append(subprocess.Popen([sys.executable, str(script)], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.STDOUT, text=True))
    outs = [p.communicate(timeout=300)[0] for p in procs]
    assert all(p.returncode == 0 for p in procs), outs
    line = [l for l in outs[0].splitlines() if l.startswith("RESULT ")][0]
    assert json.loads(line[len("RESULT "):]) == ref


SAMPLING_WORKER = r"""
import json, os, sys
sys.path.insert(0, {root!r})
import torch
from minisgl.core import SamplingParams
from minisgl.llm import LLM
prompts = json.loads(os.environ["TP_PROMPTS"])
specs = json.loads(os.environ["TP_SPECS"])
llm = LLM({path!r}, dtype=torch.float32, device="cpu", max_running_req=16)
res = []
for spec in specs:
    sps = [SamplingParams(max_tokens=10, ignore_eos=True, **s) for s in spec]
    res.append([o["token_ids"] for o in llm.generate(prompts, sps)])
if int(os.environ["RANK"]) == 0:
    print("RESULT " + json.dumps(res), flush=True)
llm.shutdown()
"""


def test_tp2_sampling_matches_tp1(tmp_path, free_port):
    """Sampled decoding under vocabulary parallelism draws the TP1 tokens in each combine mode:
    temperature only (per-shard draws, score/id pairs exchanged), top-k (+ top-p) (per-shard
    candidate lists), greedy rows mixed with top-k rows, and top-p alone (full logits gathered)."""
    from minisgl.llm import LLM

    path = make_checkpoint("tiny-qwen3", str(tmp_path / "m"))
    prompts = _prompts()
    n = len(prompts)
    specs = [
        [dict(temperature=0.8)] * n,
        [dict(temperature=0.9, top_k=20, top_p=0.9)] * n,
        [dict(temperature=0.0) if i % 2 else dict(temperature=1.1, top_k=5) for i in range(n)],
        [dict(temperature=0.7, top_p=0.8)] * n,
    ]
    llm = LLM(path, dtype=torch.float32, device="cpu", max_running_req=16, distributed_port=free_port)
    try:
        ref = []
        for spec in specs:
            sps = [SamplingParams(max_tokens=10, ignore_eos=True, **s) for s in spec]
            ref.append([o["token_ids"] for o in llm.generate(prompts, sps)])
    finally:
        llm.shutdown()
    script = tmp_path / "worker.py"
    script.write_text(SAMPLING_WORKER.format(root=ROOT, path=path))
    procs = []
    for r in range(2):
        env = dict(os.environ, RANK=str(r), LOCAL_RANK=str(r), WORLD_SIZE="2", MASTER_ADDR="127.0.0.1",
                   MASTER_PORT=str(free_port + 9), TP_PROMPTS=json.dumps(prompts), TP_SPECS=json.dumps(specs),
                   PYTHONPATH=ROOT)
        procs.append(subprocess.Popen([sys.executable, str(script)], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.STDOUT, text=True))
    outs = [p.communicate(timeout=300)[0] for p in procs]
    assert all(p.returncode == 0 for p in procs), outs
    line = [l for l in outs[0].splitlines() if l.startswith("RESULT ")][0]
    got = json.loads(line[len("RESULT "):])
    for mode, a, b in zip(("temperature", "topk", "greedy+topk", "full"), got, ref):
        assert a == b, mode


@pytest.mark.parametrize("preset,moe_parallel", [("tiny-qwen3", "tp"), ("tiny-qwen2", "tp"), ("tiny-gpt-oss", "ep")])
def test_tp4_replicates_kv_heads(tmp_path, free_port, preset, moe_parallel):
    """Four ranks for models with two KV heads: each rank keeps a replica of the KV head its
    query heads use (the reference's rule when tp > kv heads), with k/v biases and attention sinks
    for gpt-oss and two whole experts per rank under expert parallelism; tokens equal TP1."""
    from minisgl.llm import LLM

    fmt = "fused" if preset == "tiny-gpt-oss" else "per_expert"
    path = make_checkpoint(preset, str(tmp_path / "m"), expert_format=fmt)
    assert json.load(open(os.path.join(path, "config.json")))["num_key_value_heads"] < 4
    prompts = _prompts()
    llm = LLM(path, dtype=torch.float32, device="cpu", max_running_req=16, distributed_port=free_port,
              max_extend_tokens=48)
    try:
        ref = [o["token_ids"] for o in llm.generate(prompts, SamplingParams(max_tokens=12, ignore_eos=True))]
    finally:
        llm.shutdown()
    script = tmp_path / "worker.py"
    script.write_text(WORKER.format(root=ROOT, path=path))
    procs = []
    for r in range(4):
        env = dict(os.environ, RANK=str(r), LOCAL_RANK=str(r), WORLD_SIZE="4", MASTER_ADDR="127.0.0.1",
                   MASTER_PORT=str(free_port + 13), TP_PROMPTS=json.dumps(prompts), PYTHONPATH=ROOT,
                   MINISGL_MOE_PARALLEL=moe_parallel)
        procs.append(subprocess.Popen([sys.executable, str(script)], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.STDOUT, text=True))
    outs = [p.communicate(timeout=300)[0] for p in procs]
    assert all(p.returncode == 0 for p in procs), outs
    line = [l for l in outs[0].splitlines() if l.startswith("RESULT ")][0]
    assert json.loads(line[len("RESULT "):]) == ref
