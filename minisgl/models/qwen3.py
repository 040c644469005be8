"""Qwen3: QK RMSNorm per head, no biases (reference: python/minisgl/models/qwen3.py)."""

from .utils import DecoderForCausalLM


class Qwen3ForCausalLM(DecoderForCausalLM):
    layer_kwargs = dict(qk_norm=True)


__all__ = ["Qwen3ForCausalLM"]
