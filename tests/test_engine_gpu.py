"""End-to-end engine on the GPU: the bf16 sm_100a path against the fp32 CPU oracle, and
CUDA-graph / overlap scheduling against plain eager execution."""

import pytest
import torch

from minisgl.core import SamplingParams
from minisgl.models.synthetic import make_checkpoint

pytestmark = pytest.mark.gpu


def _prompts(n, vocab, seed=0, lo=16, hi=64):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, vocab, (int(torch.randint(lo, hi + 1, (1,), generator=g)),), generator=g).tolist()
            for _ in range(n)]


def _run(path, prompts, sp, port, **kw):
    from minisgl.llm import LLM

    llm = LLM(path, distributed_port=port, **kw)
    try:
        out = [o["token_ids"] for o in llm.generate(prompts, sp)]
        llm.cache_manager.check_integrity()
        from minisgl._native import cuda

        if llm.engine.is_cuda:
            code, info = cuda().get_error()
            assert code == 0, (code, info)
    finally:
        llm.shutdown()
    return out


@pytest.mark.parametrize("preset", ["tiny-qwen3", "tiny-llama", "tiny-qwen2", "tiny-qwen3-moe"])
def test_gpu_first_tokens_match_oracle(tmp_path, preset, free_port):
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    path = make_checkpoint(preset, str(tmp_path / preset), dtype=torch.bfloat16)
    prompts = _prompts(16, 1024)
    sp = SamplingParams(max_tokens=1, ignore_eos=True)
    gpu = _run(path, prompts, sp, free_port, dtype=torch.bfloat16, max_running_req=32, num_page_override=4096)
    cpu = _run(path, prompts, sp, free_port + 1, dtype=torch.float32, device="cpu", max_running_req=32)
    agree = sum(a == b for a, b in zip(gpu, cpu)) / len(gpu)
    assert agree >= 0.8, (gpu, cpu)


def test_graphs_and_overlap_are_consistent(tmp_path, free_port, monkeypatch):
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from minisgl.env import ENV

    path = make_checkpoint("tiny-qwen3", str(tmp_path / "m"), dtype=torch.bfloat16)
    prompts = _prompts(24, 1024, seed=1)
    sp = SamplingParams(max_tokens=24, ignore_eos=True)
    kw = dict(dtype=torch.bfloat16, max_running_req=32, num_page_override=8192)
    a = _run(path, prompts, sp, free_port, cuda_graph_max_bs=32, **kw)
    monkeypatch.setattr(ENV, "DISABLE_OVERLAP_SCHEDULING", True)
    b = _run(path, prompts, sp, free_port + 1, cuda_graph_max_bs=0, **kw)
    assert a == b
    # chunked prefill + radix cache hits on a repeated workload keep the same greedy tokens
    c = _run(path, prompts + prompts[:4], sp, free_port + 2, cuda_graph_max_bs=8, max_extend_tokens=64, **kw)
    assert c[:24] == a and c[24:] == a[:4]
