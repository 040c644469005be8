"""Paged KV pool for multi-head / grouped-query attention.

Layout (this engine's): one allocation ``[2, layers, slots, kv_heads, head_dim]``; a *slot* is one
token, and a page is ``page_size`` consecutive slots. Each layer's K (V) is a dense
``[slots, kv_heads * head_dim]`` matrix, so attention kernels gather 16-byte aligned rows through
the token-granular page table (reference pool: python/minisgl/kvcache/mha_pool.py:10-68).
"""

from __future__ import annotations

import torch

from minisgl import ops

from .base import BaseKVCachePool


class MHAKVCache(BaseKVCachePool):
    def __init__(
        self,
        num_kv_heads: int,
        num_layers: int,
        head_dim: int,
        num_pages: int,
        page_size: int,
        dtype: torch.dtype,
        device: torch.device,
    ):
        from minisgl.parallel import get_tp_info
        from minisgl.utils import div_even

        tp = get_tp_info()
        self.local_kv_heads = div_even(num_kv_heads, tp.size, allow_replicate=True)
        self.head_dim = head_dim
        self.page_size = page_size
        self.num_slots = num_pages * page_size
        self._buf = torch.zeros(
            (2, num_layers, self.num_slots, self.local_kv_heads, head_dim), dtype=dtype, device=device
        )
        self._k = self._buf[0]
        self._v = self._buf[1]
        self._num_layers = num_layers

    def k_cache(self, layer_id: int) -> torch.Tensor:
        return self._k[layer_id]

    def v_cache(self, layer_id: int) -> torch.Tensor:
        return self._v[layer_id]

    def store_kv(self, k: torch.Tensor, v: torch.Tensor, out_loc: torch.Tensor, layer_id: int) -> None:
        ops.store_kv(k, v, self._k[layer_id], self._v[layer_id], out_loc)

    @property
    def device(self) -> torch.device:
        return self._buf.device

    @property
    def dtype(self) -> torch.dtype:
        return self._buf.dtype

    @property
    def num_layers(self) -> int:
        return self._num_layers

    @property
    def bytes_per_token(self) -> int:
        return 2 * self._num_layers * self.local_kv_heads * self.head_dim * self._buf.element_size()
