"""Qwen2: biased QKV projection (reference: python/minisgl/models/qwen2.py)."""

from .utils import DecoderForCausalLM


class Qwen2ForCausalLM(DecoderForCausalLM):
    layer_kwargs = dict(attn_bias=True)


__all__ = ["Qwen2ForCausalLM"]
