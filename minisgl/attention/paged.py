"""This engine's paged-KV attention backend.

Prefill runs the ragged causal kernel (queries of request ``b`` are the last ``q_len[b]``
positions of its ``kv_len[b]``-long sequence, which covers prefix-cache hits and chunked prefill).
Decode with a page size of 16, 32 or 64 tokens runs the persistent paged kernel: the host cuts every
request's keys into chunks of 64-key blocks, sorts the chunks longest first and uploads that work
list with the batch; CTAs stream whole pages with TMA and the last chunk of a request to finish
combines the partials. Other page sizes run the split-KV kernel plus a combine step. Sliding
windows and per-head attention sinks are kernel arguments.

The metadata is small and device-resident: ``rows`` (page-table row per request), ``kv_lens``,
``cu_q`` and the decode work list. Decode metadata lives in static buffers so CUDA graphs replay
with fresh lengths.

Reference: python/minisgl/attention/trtllm.py (the B200 backend: paged decode/prefill over
page sizes 16/32/64), python/minisgl/attention/fi.py (split-KV decode planning).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List

import numpy as np
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
    # paged decode: work list, partial workspace and arrival counters
    work: torch.Tensor | None = None
    n_work: torch.Tensor | None = None
    ws: torch.Tensor | None = None
    ws_slots: int = 0
    counters: torch.Tensor | None = None

    def get_last_indices(self, bs: int) -> torch.Tensor:
        return (self.cu_q[1 : bs + 1] - 1).long()


PAGED_DECODE_PAGES = (16, 32, 64)


def decode_work_list(kv_lens: np.ndarray, kv_heads: int, num_ctas: int, max_entries: int | None = None):
    """Chunk every request's keys into runs of whole 64-key blocks and sort the chunks longest first.

    Returns (work int32 [n * 8], n): entry = (request, first block, end block, chunk index,
    chunks of the request, first partial slot of the request, 0, 0). The chunk length is the
    average load of one CTA (at least 4 blocks): longest-first snake order then balances the CTAs,
    and only requests longer than that pay for partials and a combine. It grows until the entries
    fit ``max_entries`` (partial slots) and a request has at most 128 chunks."""
    nblk = (kv_lens.astype(np.int64) + 63) // 64
    bs = len(nblk)
    total = int(nblk.sum())
    chb = max(4, -(-total * kv_heads // max(1, num_ctas)))
    if bs:
        chb = max(chb, -(-int(nblk.max()) // 128))  # at most 128 chunks per request (combine scratch)
    while True:
        nch = (nblk + chb - 1) // chb
        n = int(nch.sum())
        if max_entries is None or n <= max_entries or chb >= 1 << 20:
            break
        chb *= 2
    slot0 = np.zeros(bs, np.int64)
    if bs > 1:
        np.cumsum(nch[:-1], out=slot0[1:])
    b = np.repeat(np.arange(bs), nch)
    j = np.arange(n) - np.repeat(slot0, nch)
    blk0 = j * chb
    blk1 = np.minimum(blk0 + chb, nblk[b])
    order = np.argsort(blk0 - blk1, kind="stable")  # longest first
    w = np.zeros((n, 8), np.int32)
    w[:, 0] = b[order]
    w[:, 1] = blk0[order]
    w[:, 2] = blk1[order]
    w[:, 3] = j[order]
    w[:, 4] = nch[b[order]]
    w[:, 5] = slot0[b[order]]
    return w.reshape(-1), n


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
        # paged decode needs TMA-sized pages and a group of at most 16 query heads
        self.page = 0
        self.num_ctas = NUM_SMS
        if device.type == "cuda":
            ps = get_global_ctx().page_size
            if ps in PAGED_DECODE_PAGES and head_dim in (64, 128) and self.nq // self.nkv <= 16:
                self.page = ps
                self.num_ctas = _cuda().num_sms()
        self._eager: Dict[str, torch.Tensor] = {}

    def _paged_buffers(self, entries: int, bs: int, store: Dict[str, torch.Tensor]) -> None:
        """Partial workspace for `entries` chunk slots and zeroed counters for `bs` requests."""
        g = self.nq // self.nkv
        need_ws = entries * self.nkv * g * (self.hd + 2)
        if "ws" not in store or store["ws"].numel() < need_ws:
            store["ws"] = torch.empty(max(need_ws, 1), dtype=torch.float32, device=self.device)
        if "counters" not in store or store["counters"].numel() < bs * self.nkv:
            store["counters"] = torch.zeros(max(bs, 256) * self.nkv, dtype=torch.int32, device=self.device)

    def _max_entries(self, bs: int) -> int:
        return bs + 4 * self.num_ctas

    def plan_arrays(self, batch: Batch, kv_lens: np.ndarray) -> Dict[str, np.ndarray]:
        """Host-built arrays to upload with the batch (the paged decode work list)."""
        if not (self.page and batch.is_decode):
            return {}
        work, n = decode_work_list(kv_lens, self.nkv, self.num_ctas, self._max_entries(len(kv_lens)))
        return {"attn_work": work, "attn_nwork": np.array([n], np.int32)}

    # ------------------------------------------------------------------ metadata
    def prepare_metadata(self, batch: Batch, host: dict) -> None:
        dev = host["dev"]  # device views of the packed upload
        m = PagedMetadata(
            rows=dev["req_rows"],
            kv_lens=dev["kv_lens"],
            cu_q=dev["cu_q"],
            max_q_len=host["max_q_len"],
            max_kv_len=host["max_kv_len"],
            is_decode=batch.is_decode,
            num_splits=decode_splits(batch.padded_size, self.nkv, host["max_kv_len"]) if batch.is_decode else 1,
        )
        if "attn_work" in dev:
            m.work, m.n_work = dev["attn_work"], dev["attn_nwork"]
            bs = batch.padded_size
            self._paged_buffers(self._max_entries(bs), bs, self._eager)
            m.ws, m.counters = self._eager["ws"], self._eager["counters"]
            m.ws_slots = self._eager["ws"].numel() // (self.nkv * (self.nq // self.nkv) * (self.hd + 2))
        batch.attn_metadata = m

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
        if self.page:
            ent = self._max_entries(mx)
            self._graph_bufs["work"] = torch.zeros(ent * 8, **i32)
            self._graph_bufs["n_work"] = torch.zeros(1, **i32)  # nothing to do until replay
            store: Dict[str, torch.Tensor] = {}
            self._paged_buffers(ent, mx, store)
            self._graph_bufs["ws"], self._graph_bufs["counters"] = store["ws"], store["counters"]
            self._graph_ws_slots = ent

    def prepare_for_capture(self, batch: Batch) -> None:
        bs = batch.padded_size
        b = self._graph_bufs
        batch.attn_metadata = PagedMetadata(
            rows=b["rows"][:bs], kv_lens=b["kv_lens"][:bs], cu_q=b["cu_q"][: bs + 1],
            max_q_len=1, max_kv_len=self._graph_max_len, is_decode=True,
            num_splits=self._graph_splits[bs],
        )
        if self.page:
            m = batch.attn_metadata
            m.work, m.n_work, m.ws, m.counters = b["work"], b["n_work"], b["ws"], b["counters"]
            m.ws_slots = self._graph_ws_slots

    def prepare_for_replay(self, batch: Batch) -> None:
        bs = batch.padded_size
        m: PagedMetadata = batch.attn_metadata
        b = self._graph_bufs
        b["rows"][:bs].copy_(m.rows, non_blocking=True)
        b["kv_lens"][:bs].copy_(m.kv_lens, non_blocking=True)
        if self.page:
            b["work"][: m.work.numel()].copy_(m.work, non_blocking=True)
            b["n_work"].copy_(m.n_work, non_blocking=True)

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
        if m.is_decode and m.work is not None:
            _cuda().attention_decode_paged(o, q, kc, vc, ctx.page_table, m.rows, m.kv_lens, m.work, m.n_work,
                                           m.ws, m.ws_slots, m.counters, self.scale, window, sinks, self.page)
        elif m.is_decode:
            t = q.shape[0]
            ws = self._workspace(t * self.nq * m.num_splits * (self.hd + 2) * 4)
            _cuda().attention_decode(o, q, kc, vc, ctx.page_table, m.rows, m.kv_lens, self.scale,
                                     window, sinks, m.num_splits, ws)
        elif self.page and self.hd == 128:
            _cuda().attention_prefill_fmha(o, q, kc, vc, ctx.page_table, m.rows, m.cu_q, m.kv_lens, m.max_q_len,
                                           self.scale, window, sinks, self.page)
        else:
            _cuda().attention_prefill(o, q, kc, vc, ctx.page_table, m.rows, m.cu_q, m.kv_lens,
                                      m.max_q_len, self.scale, window, sinks)
        return o.view(q.shape[0], -1)
