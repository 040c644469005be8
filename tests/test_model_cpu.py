"""CPU oracle: the engine's reference path vs Hugging Face transformers on identical random
weights (greedy tokens must match exactly), for each supported dense/MoE family."""

import json
import os

import pytest
import torch

from minisgl.core import SamplingParams
from minisgl.models.synthetic import make_checkpoint


def _prompts(n=8, vocab=1000, seed=0, shared_prefix=16):
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


@pytest.mark.parametrize("preset", ["tiny-qwen3", "tiny-llama", "tiny-qwen2", "tiny-qwen3-moe", "tiny-gpt-oss",
                                    "tiny-qwen3-odd"])
def test_greedy_matches_hf(tmp_path, preset, free_port):
    """gpt-oss: checkpoint in its own fused-expert layout (what transformers loads); covers biased
    attention with sinks, alternating sliding-window layers, YaRN RoPE, top-k-then-softmax routing
    and the clamped SwiGLU experts."""
    from minisgl.llm import LLM

    fmt = "fused" if preset == "tiny-gpt-oss" else "per_expert"
    path = make_checkpoint(preset, str(tmp_path / preset), expert_format=fmt)
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


@pytest.mark.parametrize("tp", [1, 2])
def test_gpt_oss_mxfp4_checkpoint_loads_like_dequantized(tmp_path, tp):
    """MXFP4 experts (e2m1 blocks + e8m0 scales) load to exactly the tensors of the same values
    stored in the fused bf16 layout and in per-expert keys, on every TP rank."""
    from safetensors.torch import save_file

    from minisgl.models.synthetic import _gpt_oss_fused_experts, hf_config, quant_mxfp4, random_state_dict
    from minisgl.models.weight import dequant_mxfp4, load_weight
    from minisgl.parallel import set_tp_info
    from minisgl.parallel.info import reset_tp_info

    base = random_state_dict("tiny-gpt-oss")
    for k in list(base):  # snap expert weights to MXFP4-representable values
        if ".experts." in k and k.endswith(("gate_proj.weight", "up_proj.weight", "down_proj.weight")):
            base[k] = dequant_mxfp4(*quant_mxfp4(base[k]), torch.float32)
    ne = hf_config("tiny-gpt-oss")["num_local_experts"]
    layers = hf_config("tiny-gpt-oss")["num_hidden_layers"]
    dirs = {}
    for fmt in ("per_expert", "fused", "mxfp4"):
        sd = {k: v for k, v in base.items() if ".experts." not in k}
        for i in range(layers):
            p = f"model.layers.{i}."
            layer = {k: v for k, v in base.items() if k.startswith(p + "mlp.experts.")}
            sd.update(layer if fmt == "per_expert" else _gpt_oss_fused_experts(layer, p, ne, fmt, torch.float32))
        d = make_checkpoint("tiny-gpt-oss", str(tmp_path / fmt), weights=False)
        save_file({k: v.contiguous() for k, v in sd.items()}, str(tmp_path / fmt / "model.safetensors"))
        dirs[fmt] = d
    from minisgl.env import ENV

    def decoded(d):
        """Loaded tensors with MXFP4 pairs kept by the loader (``<proj>_blocks`` / ``_scales``)
        dequantised, as the MoE layer does off the GPU."""
        out = dict(load_weight(d, torch.device("cpu")))
        for k in [k for k in out if k.endswith("_blocks")]:
            base = k[: -len("_blocks")]
            out[base] = dequant_mxfp4(out.pop(k), out.pop(base + "_scales"), torch.float32)
        return {k: v.float() for k, v in out.items()}

    for keep in (True, False):
        ENV.MXFP4_RESIDENT = keep
        try:
            for rank in range(tp):
                set_tp_info(rank, tp)
                try:
                    loaded = {f: decoded(d) for f, d in dirs.items()}
                finally:
                    reset_tp_info()
                ref = loaded["per_expert"]
                for f in ("fused", "mxfp4"):
                    assert loaded[f].keys() == ref.keys(), f
                    for k in ref:
                        assert torch.equal(loaded[f][k], ref[k]), (f, k, rank, keep)
        finally:
            ENV.reload()


def test_mistral3_layout_loads_like_the_text_model(tmp_path, free_port):
    """A Mistral3 (vision-language) checkpoint: the text model's config nested under
    ``text_config``, its weights under ``language_model.``, plus vision weights that are skipped.
    It must load and generate exactly like the same weights in the plain text-model layout."""
    import shutil

    import safetensors.torch as st

    from minisgl.llm import LLM

    src = make_checkpoint("tiny-llama", str(tmp_path / "llama"))
    dst = tmp_path / "mistral3"
    shutil.copytree(src, dst)
    cfg = json.load(open(os.path.join(src, "config.json")))
    text = {k: v for k, v in cfg.items() if k not in ("architectures", "rope_scaling")}
    text["model_type"] = "mistral"
    json.dump({"architectures": ["Mistral3ForConditionalGeneration"], "model_type": "mistral3",
               "text_config": text, "torch_dtype": cfg.get("torch_dtype", "float32")},
              open(dst / "config.json", "w"))
    plain = dict(cfg, architectures=["MistralForCausalLM"], model_type="mistral")
    plain.pop("rope_scaling", None)
    json.dump(plain, open(os.path.join(src, "config.json"), "w"))
    for f in os.listdir(dst):
        if f.endswith(".safetensors"):
            tensors = st.load_file(str(dst / f))
            out = {f"language_model.{k}": v for k, v in tensors.items()}
            out["vision_tower.patch_conv.weight"] = torch.zeros(4, 3, 2, 2)
            out["multi_modal_projector.linear_1.weight"] = torch.zeros(4, 4)
            st.save_file(out, str(dst / f))
    prompts = [[1, 2, 3, 4, 5], [9, 8, 7]]
    outs = []
    for i, p in enumerate((src, str(dst))):
        llm = LLM(p, dtype=torch.float32, device="cpu", max_running_req=4, distributed_port=free_port + 3 * i)
        try:
            outs.append([o["token_ids"] for o in llm.generate(prompts, SamplingParams(max_tokens=6, ignore_eos=True))])
        finally:
            llm.shutdown()
    assert outs[0] == outs[1]
