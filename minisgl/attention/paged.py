"""This engine's paged-KV attention backend.

Prefill runs the ragged causal kernel (queries of request ``b`` are the last ``q_len[b]``
positions of its ``kv_len[b]``-long sequence, which covers prefix-cache hits and chunked prefill).
Decode runs the split-KV kernel with the GQA group packed into one tile, plus a combine step.
Sliding windows and per-head attention sinks are kernel arguments.

The metadata is small and device-resident: ``rows`` (page-table row per request), ``kv_lens``,
``cu_q``. Decode metadata lives in static buffers so CUDA graphs replay with fresh lengths.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List

import torch

from minisgl._native import cuda as _cuda
from minisgl.core import Batch, get_global_ctx
from minisgl.ops import reference as ref

from .base import BaseAttnBackend, BaseAttnMetadata

NUM_SMS = 148


@dataclass
class PagedMetadata(BaseAttnMetadata):
    rows: torch.Tensor  # [B] int32
    kv_lens: torch.Tensor  # [B] int32
    cu_q: torch.Tensor  # [B+1] int32
    max_q_len: int
    max_kv_len: int
    is_decode: bool
    num_splits: int = 1

    def get_last_indices(self, bs: int) -> torch.Tensor:
        return (self.cu_q[1 : bs + 1] - 1).long()


def decode_splits(bs: int, kv_heads: int, max_len: int, chunk: int = 256) -> int:
    """Split the KV axis so that about two waves of CTAs cover the GPU, without splitting below
    one ``chunk`` of keys per split."""
    ctas = max(bs * kv_heads, 1)
    want = max(1, (2 * NUM_SMS + ctas - 1) // ctas)
    return max(1, min(want, (max_len + chunk - 1) // chunk, 64))


class PagedAttentionBackend(BaseAttnBackend):
    def __init__(self, num_qo_heads: int, num_kv_heads: int, head_dim: int, device: torch.device):
        from minisgl.parallel import get_tp_info
        from minisgl.utils import div_even

        tp = get_tp_info().size
        self.nq = div_even(num_qo_heads, tp)
        self.nkv = div_even(num_kv_heads, tp, allow_replicate=True)
        self.hd = head_dim
        self.device = device
        self.scale = ref.softmax_scale(head_dim)
        self._graph_bufs: Dict[str, torch.Tensor] | None = None
        self._graph_splits: Dict[int, int] = {}
        self._ws: torch.Tensor | None = None

    # ------------------------------------------------------------------ metadata
    def prepare_metadata(self, batch: Batch, host: dict) -> None:
        dev = host["dev"]  # device views of the packed upload
        batch.attn_metadata = PagedMetadata(
            rows=dev["req_rows"],
            kv_lens=dev["kv_lens"],
            cu_q=dev["cu_q"],
            max_q_len=host["max_q_len"],
            max_kv_len=host["max_kv_len"],
            is_decode=batch.is_decode,
            num_splits=decode_splits(batch.padded_size, self.nkv, host["max_kv_len"]) if batch.is_decode else 1,
        )

    def init_capture_graph(self, max_seq_len: int, bs_list: List[int]) -> None:
        mx = max(bs_list)
        i32 = dict(dtype=torch.int32, device=self.device)
        self._graph_bufs = {
            "rows": torch.zeros(mx, **i32),
            "kv_lens": torch.ones(mx, **i32),
            "cu_q": torch.arange(mx + 1, **i32),
        }
        self._graph_max_len = max_seq_len
        for bs in bs_list:
            self._graph_splits[bs] = decode_splits(bs, self.nkv, max_seq_len)

    def prepare_for_capture(self, batch: Batch) -> None:
        bs = batch.padded_size
        b = self._graph_bufs
        batch.attn_metadata = PagedMetadata(
            rows=b["rows"][:bs], kv_lens=b["kv_lens"][:bs], cu_q=b["cu_q"][: bs + 1],
            max_q_len=1, max_kv_len=self._graph_max_len, is_decode=True,
            num_splits=self._graph_splits[bs],
        )

    def prepare_for_replay(self, batch: Batch) -> None:
        bs = batch.padded_size
        m: PagedMetadata = batch.attn_metadata
        b = self._graph_bufs
        b["rows"][:bs].copy_(m.rows, non_blocking=True)
        b["kv_lens"][:bs].copy_(m.kv_lens, non_blocking=True)

    # ------------------------------------------------------------------ compute
    def _workspace(self, nbytes: int) -> torch.Tensor:
        if self._ws is None or self._ws.numel() < nbytes:
            self._ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=self.device)
        return self._ws

    def forward(self, q: torch.Tensor, layer_id: int, batch: Batch, *, window: int = -1,
                sinks: torch.Tensor | None = None) -> torch.Tensor:
        ctx = get_global_ctx()
        kc, vc = ctx.kv_cache.k_cache(layer_id), ctx.kv_cache.v_cache(layer_id)
        m: PagedMetadata = batch.attn_metadata
        if not q.is_cuda:
            o = ref.paged_attention(q, kc, vc, ctx.page_table, m.rows, m.cu_q, m.kv_lens,
                                    self.scale, window, sinks)
            return o.reshape(q.shape[0], -1)
        o = torch.empty_like(q)
        if m.is_decode:
            t = q.shape[0]
            ws = self._workspace(t * self.nq * m.num_splits * (self.hd + 2) * 4)
            _cuda().attention_decode(o, q, kc, vc, ctx.page_table, m.rows, m.kv_lens, self.scale,
                                     window, sinks, m.num_splits, ws)
        else:
            _cuda().attention_prefill(o, q, kc, vc, ctx.page_table, m.rows, m.cu_q, m.kv_lens,
                                      m.max_q_len, self.scale, window, sinks)
        return o.view(q.shape[0], -1)
