"""Failure detection and overload behaviour, on the host only (no GPU is faulted, trapped or hung):

* a tensor-parallel rank that exits, or stops answering (SIGSTOP), between steps: the surviving
  rank's next collective must raise within the process-group timeout instead of waiting forever;
* a KV pool far smaller than the offered load: requests wait for pages (admission backpressure)
  and every one of them completes with the tokens of an unconstrained run.
"""

import json
import os
import signal
import subprocess
import sys
import time

import pytest
import torch

from minisgl.core import SamplingParams
from minisgl.models.synthetic import make_checkpoint

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

WORKER = r"""
import os, signal, sys, time
sys.path.insert(0, {root!r})
import torch
from minisgl.core import SamplingParams
from minisgl.llm import LLM
rank = int(os.environ["RANK"])
llm = LLM({path!r}, dtype=torch.float32, device="cpu", max_running_req=8, distributed_timeout=5.0)
print("READY", rank, flush=True)
if rank == 1:
    if {mode!r} == "exit":
        os._exit(3)  # leaves between steps: nothing of it is in flight
    os.kill(os.getpid(), signal.SIGSTOP)  # stops answering; the test kills it afterwards
t0 = time.time()
try:
    llm.generate([[1, 2, 3, 4]], SamplingParams(max_tokens=4, ignore_eos=True))
except Exception as e:  # the collective with the missing rank must fail, not hang
    print("RAISED %.1f %s" % (time.time() - t0, type(e).__name__), flush=True)
    os._exit(7)
print("NO ERROR", flush=True)
os._exit(0)
"""


@pytest.mark.parametrize("mode", ["exit", "stop"])
def test_lost_tp_rank_raises_within_timeout(tmp_path, free_port, mode):
    path = make_checkpoint("tiny-qwen3", str(tmp_path / "m"))
    script = tmp_path / "worker.py"
    script.write_text(WORKER.format(root=ROOT, path=path, mode=mode))
    procs = []
    for r in range(2):
        env = dict(os.environ, RANK=str(r), LOCAL_RANK=str(r), WORLD_SIZE="2", MASTER_ADDR="127.0.0.1",
                   MASTER_PORT=str(free_port + 11), PYTHONPATH=ROOT)
        procs.append(subprocess.Popen([sys.executable, str(script)], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.STDOUT, text=True))
    t0 = time.time()
    try:
        out0 = procs[0].communicate(timeout=180)[0]
    finally:
        if procs[1].poll() is None:  # the stopped rank: kill exactly that process
            os.kill(procs[1].pid, signal.SIGKILL)
        procs[1].communicate(timeout=60)
    assert "READY 0" in out0, out0
    assert procs[0].returncode == 7, out0
    raised = [l for l in out0.splitlines() if l.startswith("RAISED")]
    assert raised and float(raised[0].split()[1]) < 60.0, out0
    assert time.time() - t0 < 170


@pytest.mark.parametrize("page,pages", [(1, 96), (16, 8)])
def test_small_kv_pool_backpressure(tmp_path, free_port, page, pages):
    """Pages are allocated whole: admission reserves a partial page per request, so a tight pool
    never runs dry mid-decode (8 pages of 16 hold about one request at a time here)."""
    from minisgl.llm import LLM

    path = make_checkpoint("tiny-qwen3", str(tmp_path / "m"))
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, 1024, (int(torch.randint(20, 60, (1,), generator=g)),), generator=g).tolist()
               for _ in range(12)]
    sp = SamplingParams(max_tokens=16, ignore_eos=True)
    outs = {}
    for name, npages in (("roomy", None), ("tight", pages)):
        llm = LLM(path, dtype=torch.float32, device="cpu", max_running_req=8, page_size=page,
                  num_page_override=npages, distributed_port=free_port + (0 if npages is None else 3),
                  cache_type="radix")
        try:
            outs[name] = [o["token_ids"] for o in llm.generate(prompts, sp)]
            llm.cache_manager.check_integrity()
        finally:
            llm.shutdown()
    assert all(len(o) == 16 for o in outs["tight"])
    assert outs["tight"] == outs["roomy"], json.dumps(outs)
