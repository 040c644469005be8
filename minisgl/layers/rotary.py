"""Rotary position embedding tables (reference: python/minisgl/layers/rotary.py:12-143).

Only the fp32 ``[max_pos, rotary_dim]`` table ``[cos | sin]`` lives here; the rotation itself is
fused into the QK-norm + RoPE + KV-store kernel. Scaling types: default, llama3, yarn.
"""

from __future__ import annotations

import functools
import math
from typing import Any, Dict, Tuple

import torch

from minisgl.ops import reference as ref

_ROPE_DEVICE: torch.device | None = None


def set_rope_device(device: torch.device | str) -> None:
    global _ROPE_DEVICE
    _ROPE_DEVICE = torch.device(device)


class RotaryEmbedding:
    def __init__(self, head_dim: int, rotary_dim: int, max_position: int, inv_freq: torch.Tensor,
                 attention_factor: float = 1.0):
        assert rotary_dim == head_dim, "partial rotary is not used by the supported models"
        self.head_size = head_dim
        table = ref.rope_cos_sin(max_position, rotary_dim, inv_freq) * attention_factor
        device = _ROPE_DEVICE if _ROPE_DEVICE is not None else torch.device("cpu")
        self.cos_sin_cache = table.to(device)


def _llama3(inv_freq: torch.Tensor, s: Dict[str, Any]) -> torch.Tensor:
    factor, lo, hi = s["factor"], s["low_freq_factor"], s["high_freq_factor"]
    orig = s["original_max_position_embeddings"]
    wave = 2 * math.pi / inv_freq
    if lo == hi:
        return torch.where(wave < orig / hi, inv_freq, inv_freq / factor)
    smooth = ((orig / wave - lo) / (hi - lo)).clamp(0, 1)
    return ((1 - smooth) / factor + smooth) * inv_freq


def _yarn(inv_freq: torch.Tensor, s: Dict[str, Any], rotary_dim: int, base: float) -> Tuple[torch.Tensor, float]:
    factor = s["factor"]
    beta_fast, beta_slow = s.get("beta_fast", 32.0), s.get("beta_slow", 1.0)
    orig = s["original_max_position_embeddings"]

    def corr_dim(rot: float) -> float:
        return rotary_dim * math.log(orig / (rot * 2 * math.pi)) / (2 * math.log(base))

    lo = max(math.floor(corr_dim(beta_fast)), 0)
    hi = min(math.ceil(corr_dim(beta_slow)), rotary_dim // 2 - 1)
    ramp = ((torch.arange(rotary_dim // 2, dtype=torch.float32) - lo) / max(hi - lo, 1)).clamp(0, 1)
    # ramp = 0 -> extrapolate (keep), 1 -> interpolate (divide by factor)
    out = (inv_freq / factor) * ramp + inv_freq * (1 - ramp)
    mscale = s.get("attention_factor")
    if mscale is None:
        mscale = 0.1 * math.log(factor) + 1.0 if factor > 1 else 1.0
    return out, float(mscale)


def get_rope(head_dim: int, rotary_dim: int, max_position: int, base: float,
             rope_scaling: Tuple[Tuple[str, Any], ...] | None = None) -> RotaryEmbedding:
    """Cached per (shape, scaling, device). Tables are built on the CPU in fp32 (even while the
    model is being constructed on the meta device) and moved to the rope device."""
    dev = str(_ROPE_DEVICE) if _ROPE_DEVICE is not None else "cpu"
    with torch.device("cpu"):
        return _get_rope(head_dim, rotary_dim, max_position, base, rope_scaling, dev)


@functools.cache
def _get_rope(head_dim: int, rotary_dim: int, max_position: int, base: float,
              rope_scaling, device: str) -> RotaryEmbedding:
    s = dict(rope_scaling) if rope_scaling else None
    inv = ref.default_inv_freq(rotary_dim, base)
    kind = (s or {}).get("rope_type", (s or {}).get("type", "default"))
    if s is None or kind == "default":
        return RotaryEmbedding(head_dim, rotary_dim, max_position, inv)
    if kind == "llama3":
        return RotaryEmbedding(head_dim, rotary_dim, max_position, _llama3(inv, s))
    if kind == "yarn":
        inv2, mscale = _yarn(inv, s, rotary_dim, base)
        return RotaryEmbedding(head_dim, rotary_dim, max_position, inv2, mscale)
    raise ValueError(f"unsupported rope scaling {s}")
