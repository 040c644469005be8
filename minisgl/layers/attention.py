"""Attention layer: QK-norm + RoPE + KV store in one fused op, then paged attention
(reference: python/minisgl/layers/attention.py:18-57)."""

from __future__ import annotations

import torch

from minisgl import ops
from minisgl.core import get_global_ctx
from minisgl.parallel import get_tp_info
from minisgl.utils import div_even

from .base import BaseOP
from .norm import RMSNorm
from .rotary import get_rope


class AttentionLayer(BaseOP):
    def __init__(self, layer_id: int, head_dim: int, num_qo_heads: int, num_kv_heads: int,
                 rotary_config, q_norm: RMSNorm | None = None, k_norm: RMSNorm | None = None,
                 sliding_window: int = -1, has_sinks: bool = False):
        tp = get_tp_info().size
        self._layer_id = layer_id
        self._hd = head_dim
        self._nq = div_even(num_qo_heads, tp)
        self._nkv = div_even(num_kv_heads, tp, allow_replicate=True)
        rc = rotary_config
        scaling = tuple(sorted(rc.scaling.items())) if rc.scaling else None
        self._rope = get_rope(head_dim, rc.rotary_dim, rc.max_position, rc.base, scaling)
        self._q_norm = q_norm
        self._k_norm = k_norm
        self._eps = q_norm.eps if q_norm is not None else 1e-6
        self._window = sliding_window
        self.sinks = torch.empty(self._nq, dtype=torch.float32) if has_sinks else None

    def forward(self, qkv: torch.Tensor) -> torch.Tensor:
        ctx = get_global_ctx()
        batch = ctx.batch
        kv = ctx.kv_cache
        q = ops.qk_norm_rope_store(
            qkv, batch.positions, self._rope.cos_sin_cache,
            self._q_norm.weight if self._q_norm is not None else None,
            self._k_norm.weight if self._k_norm is not None else None,
            self._eps, kv.k_cache(self._layer_id), kv.v_cache(self._layer_id), batch.out_loc,
            self._nq, self._nkv, self._hd,
        )
        return ctx.attn_backend.forward(q, self._layer_id, batch, window=self._window, sinks=self.sinks)
