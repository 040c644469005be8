"""Synthetic checkpoints: HF ``config.json`` + a local tokenizer + (optionally) random
N(0, std) safetensors for the architectures the benchmarks name. There is no model hub access on
the build machines, so every test and benchmark builds its model directory with this module.

``python -m minisgl.models.synthetic qwen3-0.6b /tmp/q06 [--weights]``
"""

from __future__ import annotations

import json
import os
from typing import Dict

import torch

PRESETS: Dict[str, dict] = {
    # the CPU plumbing model of the benchmark plan
    "tiny-qwen3": dict(
        architectures=["Qwen3ForCausalLM"], model_type="qwen3", num_hidden_layers=2, hidden_size=256,
        num_attention_heads=4, num_key_value_heads=2, head_dim=64, intermediate_size=512,
        vocab_size=1024, rope_theta=1e6, tie_word_embeddings=True, max_position_embeddings=4096,
    ),
    # an intermediate size whose per-rank share is not a whole gate/up interleave block, and a
    # vocabulary that does not split evenly over ranks
    "tiny-qwen3-odd": dict(
        architectures=["Qwen3ForCausalLM"], model_type="qwen3", num_hidden_layers=2, hidden_size=256,
        num_attention_heads=4, num_key_value_heads=2, head_dim=64, intermediate_size=320,
        vocab_size=1001, rope_theta=1e6, tie_word_embeddings=True, max_position_embeddings=4096,
    ),
    "tiny-llama": dict(
        architectures=["LlamaForCausalLM"], model_type="llama", num_hidden_layers=2, hidden_size=256,
        num_attention_heads=4, num_key_value_heads=2, head_dim=64, intermediate_size=512,
        vocab_size=1024, rope_theta=5e5, tie_word_embeddings=False, max_position_embeddings=4096,
        rope_scaling=dict(rope_type="llama3", factor=8.0, low_freq_factor=1.0, high_freq_factor=4.0,
                          original_max_position_embeddings=1024),
    ),
    "tiny-qwen2": dict(
        architectures=["Qwen2ForCausalLM"], model_type="qwen2", num_hidden_layers=2, hidden_size=256,
        num_attention_heads=4, num_key_value_heads=2, intermediate_size=512, vocab_size=1024,
        rope_theta=1e6, tie_word_embeddings=False, max_position_embeddings=4096,
    ),
    "tiny-qwen3-moe": dict(
        architectures=["Qwen3MoeForCausalLM"], model_type="qwen3_moe", num_hidden_layers=2,
        hidden_size=256, num_attention_heads=4, num_key_value_heads=2, head_dim=64,
        intermediate_size=512, moe_intermediate_size=128, num_experts=8, num_experts_per_tok=2,
        norm_topk_prob=True, vocab_size=1024, rope_theta=1e6, tie_word_embeddings=False,
        max_position_embeddings=4096,
    ),
    "tiny-gpt-oss": dict(
        architectures=["GptOssForCausalLM"], model_type="gpt_oss", num_hidden_layers=2,
        hidden_size=256, num_attention_heads=4, num_key_value_heads=2, head_dim=64,
        intermediate_size=128, num_local_experts=8, num_experts_per_tok=2, experts_per_token=2,
        vocab_size=1024, rope_theta=150000.0, tie_word_embeddings=False, max_position_embeddings=4096,
        sliding_window=16, layer_types=["sliding_attention", "full_attention"], attention_bias=True,
        rope_scaling=dict(rope_type="yarn", factor=32.0, beta_fast=32.0, beta_slow=1.0,
                          original_max_position_embeddings=4096, truncate=False),
    ),
    "qwen3-0.6b": dict(
        architectures=["Qwen3ForCausalLM"], model_type="qwen3", num_hidden_layers=28, hidden_size=1024,
        num_attention_heads=16, num_key_value_heads=8, head_dim=128, intermediate_size=3072,
        vocab_size=151936, rope_theta=1e6, tie_word_embeddings=True, max_position_embeddings=40960,
    ),
    "qwen3-14b": dict(
        architectures=["Qwen3ForCausalLM"], model_type="qwen3", num_hidden_layers=40, hidden_size=5120,
        num_attention_heads=40, num_key_value_heads=8, head_dim=128, intermediate_size=17408,
        vocab_size=151936, rope_theta=1e6, tie_word_embeddings=False, max_position_embeddings=40960,
    ),
    "qwen3-32b": dict(
        architectures=["Qwen3ForCausalLM"], model_type="qwen3", num_hidden_layers=64, hidden_size=5120,
        num_attention_heads=64, num_key_value_heads=8, head_dim=128, intermediate_size=25600,
        vocab_size=151936, rope_theta=1e6, tie_word_embeddings=False, max_position_embeddings=40960,
    ),
    "gpt-oss-120b": dict(
        architectures=["GptOssForCausalLM"], model_type="gpt_oss", num_hidden_layers=36,
        hidden_size=2880, num_attention_heads=64, num_key_value_heads=8, head_dim=64,
        intermediate_size=2880, num_local_experts=128, num_experts_per_tok=4, experts_per_token=4,
        vocab_size=201088, rope_theta=150000.0, tie_word_embeddings=False,
        max_position_embeddings=131072, sliding_window=128, attention_bias=True,
        layer_types=["sliding_attention", "full_attention"] * 18,
        rope_scaling=dict(rope_type="yarn", factor=32.0, beta_fast=32.0, beta_slow=1.0,
                          original_max_position_embeddings=4096, truncate=False),
        quantization_config=dict(quant_method="mxfp4"),
    ),
}

_COMMON = dict(rms_norm_eps=1e-6, hidden_act="silu", torch_dtype="bfloat16", bos_token_id=1,
               eos_token_id=2, pad_token_id=0, attention_bias=False)


def write_tokenizer(path: str, vocab_size: int) -> None:
    """A byte-level BPE tokenizer with no merges: ids 0-2 are specials, 3-258 the 256 bytes, the
    rest are filler tokens so every model id decodes to something."""
    from tokenizers import Tokenizer, decoders, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast

    specials = ["<pad>", "<s>", "</s>"]
    byte_chars = pre_tokenizers.ByteLevel.alphabet()
    vocab = {s: i for i, s in enumerate(specials)}
    for ch in sorted(byte_chars):
        vocab[ch] = len(vocab)
    i = 0
    while len(vocab) < vocab_size:
        vocab[f"<x{i}>"] = len(vocab)
        i += 1
    tok = Tokenizer(models.BPE(vocab=vocab, merges=[], unk_token=None))
    tok.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False)
    tok.decoder = decoders.ByteLevel()
    fast = PreTrainedTokenizerFast(tokenizer_object=tok, bos_token="<s>", eos_token="</s>",
                                   pad_token="<pad>")
    fast.chat_template = (
        "{% for m in messages %}<s>{{ m['role'] }}\n{{ m['content'] }}</s>\n{% endfor %}"
        "{% if add_generation_prompt %}<s>assistant\n{% endif %}"
    )
    fast.save_pretrained(path)


def hf_config(preset: str) -> dict:
    cfg = dict(_COMMON)
    cfg.update(PRESETS[preset])
    return cfg


def quant_mxfp4(w: torch.Tensor):
    """OCP MX fp4 quantisation along the last dim (a multiple of 32): per 32-value block the e8m0
    scale 2^e is the smallest power of two with max|w| / 2^e <= 6, values round to the nearest e2m1
    code. Returns (blocks [..., K/32, 16] uint8, low nibble first; scales [..., K/32] uint8, bias 127)."""
    x = w.float().reshape(*w.shape[:-1], -1, 32)
    amax = x.abs().amax(-1)
    e = torch.ceil(torch.log2(amax.clamp(min=2.0 ** -126) / 6.0)).clamp(-127, 127)
    q = x / torch.exp2(e).unsqueeze(-1)
    mags = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])
    code = (q.abs().unsqueeze(-1) - mags).abs().argmin(-1) | ((q < 0).long() << 3)
    code = code.to(torch.uint8)
    blocks = code[..., 0::2] | (code[..., 1::2] << 4)
    return blocks.contiguous(), (e + 127).to(torch.uint8).contiguous()


def _gpt_oss_fused_experts(per_expert: Dict[str, torch.Tensor], prefix: str, ne: int, fmt: str, dtype):
    """Per-expert gate/up/down (+ biases) of one layer -> the gpt-oss checkpoint layout: fused
    ``gate_up_proj [E, H, 2I]`` (gate / up interleaved) and ``down_proj [E, I, H]`` ("fused"), or
    their MXFP4 blocks / scales over the input dim ("mxfp4")."""
    q = prefix + "mlp.experts."
    g = torch.stack([per_expert[f"{q}{e}.gate_proj.weight"] for e in range(ne)]).float()  # [E, I, H]
    u = torch.stack([per_expert[f"{q}{e}.up_proj.weight"] for e in range(ne)]).float()
    d = torch.stack([per_expert[f"{q}{e}.down_proj.weight"] for e in range(ne)]).float()  # [E, H, I]
    gu = torch.stack([g, u], dim=2).reshape(ne, -1, g.shape[-1])  # rows interleaved: [E, 2I, H]
    out = {}
    if fmt == "mxfp4":
        out[q + "gate_up_proj_blocks"], out[q + "gate_up_proj_scales"] = quant_mxfp4(gu)
        out[q + "down_proj_blocks"], out[q + "down_proj_scales"] = quant_mxfp4(d)
    else:
        out[q + "gate_up_proj"] = gu.transpose(1, 2).contiguous().to(dtype)
        out[q + "down_proj"] = d.transpose(1, 2).contiguous().to(dtype)
    gb = torch.stack([per_expert[f"{q}{e}.gate_proj.bias"] for e in range(ne)])
    ub = torch.stack([per_expert[f"{q}{e}.up_proj.bias"] for e in range(ne)])
    out[q + "gate_up_proj_bias"] = torch.stack([gb, ub], dim=2).reshape(ne, -1).contiguous()
    out[q + "down_proj_bias"] = torch.stack([per_expert[f"{q}{e}.down_proj.bias"] for e in range(ne)])
    return out


def random_state_dict(preset: str, seed: int = 0, std: float = 0.02, dtype=torch.float32,
                      expert_format: str = "per_expert") -> Dict[str, torch.Tensor]:
    """HF-named random weights. MoE experts as per-expert keys, or for gpt-oss its own fused
    ("fused") or MXFP4 ("mxfp4") layout. Norm weights are ones."""
    c = hf_config(preset)
    g = torch.Generator().manual_seed(seed)
    H, L = c["hidden_size"], c["num_hidden_layers"]
    nq, nkv = c["num_attention_heads"], c["num_key_value_heads"]
    hd = c.get("head_dim") or H // nq
    V = c["vocab_size"]
    out: Dict[str, torch.Tensor] = {}

    def rnd(*shape):
        return (torch.randn(*shape, generator=g) * std).to(dtype)

    out["model.embed_tokens.weight"] = rnd(V, H)
    for i in range(L):
        p = f"model.layers.{i}."
        out[p + "input_layernorm.weight"] = torch.ones(H, dtype=dtype)
        out[p + "post_attention_layernorm.weight"] = torch.ones(H, dtype=dtype)
        out[p + "self_attn.q_proj.weight"] = rnd(nq * hd, H)
        out[p + "self_attn.k_proj.weight"] = rnd(nkv * hd, H)
        out[p + "self_attn.v_proj.weight"] = rnd(nkv * hd, H)
        out[p + "self_attn.o_proj.weight"] = rnd(H, nq * hd)
        if c["model_type"] in ("qwen2", "gpt_oss"):
            for n, d in (("q", nq), ("k", nkv), ("v", nkv)):
                out[p + f"self_attn.{n}_proj.bias"] = rnd(d * hd)
        if c["model_type"] == "gpt_oss":
            out[p + "self_attn.o_proj.bias"] = rnd(H)
            out[p + "self_attn.sinks"] = rnd(nq).float()
        if c["model_type"] in ("qwen3", "qwen3_moe"):
            out[p + "self_attn.q_norm.weight"] = torch.ones(hd, dtype=dtype)
            out[p + "self_attn.k_norm.weight"] = torch.ones(hd, dtype=dtype)
        ne = c.get("num_experts") or c.get("num_local_experts") or 0
        if ne:
            inter = c.get("moe_intermediate_size") or c["intermediate_size"]
            router = "router" if c["model_type"] == "gpt_oss" else "gate"
            out[p + f"mlp.{router}.weight"] = rnd(ne, H)
            if c["model_type"] == "gpt_oss":
                out[p + "mlp.router.bias"] = rnd(ne)
            layer_experts: Dict[str, torch.Tensor] = {}
            for e in range(ne):
                q = p + f"mlp.experts.{e}."
                layer_experts[q + "gate_proj.weight"] = rnd(inter, H)
                layer_experts[q + "up_proj.weight"] = rnd(inter, H)
                layer_experts[q + "down_proj.weight"] = rnd(H, inter)
                if c["model_type"] == "gpt_oss":
                    layer_experts[q + "gate_proj.bias"] = rnd(inter)
                    layer_experts[q + "up_proj.bias"] = rnd(inter)
                    layer_experts[q + "down_proj.bias"] = rnd(H)
            if expert_format != "per_expert" and c["model_type"] == "gpt_oss":
                out.update(_gpt_oss_fused_experts(layer_experts, p, ne, expert_format, dtype))
            else:
                out.update(layer_experts)
        else:
            I = c["intermediate_size"]
            out[p + "mlp.gate_proj.weight"] = rnd(I, H)
            out[p + "mlp.up_proj.weight"] = rnd(I, H)
            out[p + "mlp.down_proj.weight"] = rnd(H, I)
    out["model.norm.weight"] = torch.ones(H, dtype=dtype)
    if not c["tie_word_embeddings"]:
        out["lm_head.weight"] = rnd(V, H)
    return out


def make_checkpoint(preset: str, path: str, *, weights: bool = True, seed: int = 0, std: float = 0.02,
                    dtype: torch.dtype = torch.float32, expert_format: str = "per_expert") -> str:
    os.makedirs(path, exist_ok=True)
    cfg = hf_config(preset)
    cfg["torch_dtype"] = {torch.float32: "float32", torch.bfloat16: "bfloat16"}[dtype]
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg, f, indent=1)
    if not os.path.exists(os.path.join(path, "tokenizer.json")):
        write_tokenizer(path, cfg["vocab_size"])
    if weights:
        from safetensors.torch import save_file

        sd = random_state_dict(preset, seed=seed, std=std, dtype=dtype, expert_format=expert_format)
        save_file({k: v.contiguous() for k, v in sd.items()}, os.path.join(path, "model.safetensors"))
    return path


if __name__ == "__main__":
    import argparse

    ap = argparse.ArgumentParser()
    ap.add_argument("preset", choices=sorted(PRESETS))
    ap.add_argument("path")
    ap.add_argument("--weights", action="store_true")
    ap.add_argument("--bf16", action="store_true")
    ap.add_argument("--expert-format", default="per_expert", choices=["per_expert", "fused", "mxfp4"],
                    help="gpt-oss experts: per-expert keys, the fused bf16 layout or MXFP4 blocks/scales")
    a = ap.parse_args()
    make_checkpoint(a.preset, a.path, weights=a.weights, dtype=torch.bfloat16 if a.bf16 else torch.float32,
                    expert_format=a.expert_format)
