"""CPU oracle: the engine's reference path vs Hugging Face transformers on identical random
weights (greedy tokens must match exactly), for each supported dense/MoE family."""

import pytest
import torch

from minisgl.core import SamplingParams
from minisgl.models.synthetic import make_checkpoint


def _prompts(n=8, vocab=1024, seed=0, shared_prefix=16):
    g = torch.Generator().manual_seed(seed)
    prefix = torch.randint(0, vocab, (shared_prefix,), generator=g).tolist()
    out = []
    for i in range(n):
        L = int(torch.randint(16, 65, (1,), generator=g))
        p = torch.randint(0, vocab, (L,), generator=g).tolist()
        if i < 4:
            p = prefix + p[shared_prefix:] if L > shared_prefix else prefix
        out.append(p)
    return out


def _hf_greedy(path, prompts, n_new):
    from transformers import AutoModelForCausalLM

    m = AutoModelForCausalLM.from_pretrained(path, dtype=torch.float32).eval()
    outs = []
    with torch.no_grad():
        for p in prompts:
            ids = torch.tensor([p])
            for _ in range(n_new):
                nxt = int(m(ids).logits[0, -1].argmax())
                ids = torch.cat([ids, torch.tensor([[nxt]])], dim=1)
            outs.append(ids[0, len(p):].tolist())
    return outs


@pytest.mark.parametrize("preset", ["tiny-qwen3", "tiny-llama", "tiny-qwen2", "tiny-qwen3-moe"])
def test_greedy_matches_hf(tmp_path, preset, free_port):
    from minisgl.llm import LLM

    path = make_checkpoint(preset, str(tmp_path / preset))
    prompts = _prompts()
    n_new = 8
    llm = LLM(path, dtype=torch.float32, device="cpu", max_running_req=16, distributed_port=free_port,
              cache_type="radix")
    try:
        ours = [o["token_ids"] for o in llm.generate(prompts, SamplingParams(max_tokens=n_new, ignore_eos=True))]
        llm.cache_manager.check_integrity()
    finally:
        llm.shutdown()
    ref = _hf_greedy(path, prompts, n_new)
    assert ours == ref


def test_tiny_config_full_workload(tmp_path, free_port):
    """The plumbing config of the benchmark plan: 8 requests, 32 greedy tokens, radix on, requests
    0-3 share a 16-token prefix, page size 1; chunked prefill forced by a small token budget."""
    from minisgl.llm import LLM

    path = make_checkpoint("tiny-qwen3", str(tmp_path / "m"))
    prompts = _prompts()
    sp = SamplingParams(max_tokens=32, ignore_eos=True)
    llm = LLM(path, dtype=torch.float32, device="cpu", max_running_req=16, distributed_port=free_port,
              max_extend_tokens=40)
    try:
        a = [o["token_ids"] for o in llm.generate(prompts, sp)]
        # the shared prefix is served by the radix cache on a second run
        assert llm.cache_manager.prefix_cache.size_info.evictable_size > 0
        b = [o["token_ids"] for o in llm.generate(prompts, sp)]
        llm.cache_manager.check_integrity()
    finally:
        llm.shutdown()
    assert a == b
    assert all(len(x) == 32 for x in a)
    llm2 = LLM(path, dtype=torch.float32, device="cpu", max_running_req=16, distributed_port=free_port + 1,
               cache_type="naive")
    try:
        c = [o["token_ids"] for o in llm2.generate(prompts, sp)]
    finally:
        llm2.shutdown()
    assert a == c
