"""Qwen3-MoE: Qwen3 attention + routed experts (reference: python/minisgl/models/qwen3_moe.py)."""

from .utils import DecoderForCausalLM


class Qwen3MoeForCausalLM(DecoderForCausalLM):
    layer_kwargs = dict(qk_norm=True, moe=True)


__all__ = ["Qwen3MoeForCausalLM"]
