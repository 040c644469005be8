"""Gated activations (reference: python/minisgl/layers/activation.py:9-18)."""

from minisgl.ops import gelu_and_mul, silu_and_mul

__all__ = ["silu_and_mul", "gelu_and_mul"]
