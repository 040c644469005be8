"""Llama / Mistral: plain decoder (reference: python/minisgl/models/llama.py, mistral.py)."""

from .utils import DecoderForCausalLM


class LlamaForCausalLM(DecoderForCausalLM):
    layer_kwargs = dict()


class MistralForCausalLM(DecoderForCausalLM):
    layer_kwargs = dict()


__all__ = ["LlamaForCausalLM", "MistralForCausalLM"]
