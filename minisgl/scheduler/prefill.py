"""FCFS prefill admission with chunking (reference: python/minisgl/scheduler/prefill.py:23-158).

A request is admitted when its extend length plus its output budget, plus one partial page,
fits in the KV pool (free + evictable) after reserving what the running decode set and the
requests admitted before it in the batch may still claim (pages are allocated whole, so each
request can hold up to page_size - 1 slots beyond its tokens). A prompt that does not
fit the per-batch token budget becomes a ``ChunkedReq``: it is computed over several prefill
batches, is never sampled until its last chunk, and is re-queued at the head of the list.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Tuple

import numpy as np
import torch

from minisgl.core import Batch, Req
from minisgl.kvcache import BaseCacheHandle

from .cache import CacheManager
from .decode import DecodeManager
from .table import TableManager


class ChunkedReq(Req):
    def append_host(self, next_token: int) -> None:
        raise RuntimeError("a chunked request is not sampled")

    @property
    def can_decode(self) -> bool:
        return False


class Waiting:
    """A request in the prefill queue: its prompt, its output budget and, after its first chunk
    ran, the ``ChunkedReq`` that carries its page-table row, slots and cache handle to the next
    chunk."""

    __slots__ = ("uid", "input_ids", "sampling_params", "prompt_len", "budget", "chunk")

    def __init__(self, uid: int, input_ids: torch.Tensor, sampling_params) -> None:
        self.uid = uid
        self.input_ids = input_ids
        self.sampling_params = sampling_params
        self.prompt_len = int(input_ids.shape[0])
        self.budget = int(sampling_params.max_tokens)
        self.chunk: ChunkedReq | None = None


@dataclass
class PrefillAdder:
    token_budget: int
    reserved_size: int
    cache_manager: CacheManager
    table_manager: TableManager

    def _admit(self, p: Waiting) -> Tuple[BaseCacheHandle, int, np.ndarray] | None:
        if self.table_manager.available_size == 0:
            return None
        handle = self.cache_manager.match_req(p.input_ids).cuda_handle
        need = p.prompt_len - handle.cached_len + p.budget + self.cache_manager.page_size - 1
        if need + self.reserved_size > self.cache_manager.available_size:
            return None
        self.cache_manager.lock(handle)  # locking moves the match out of the evictable pool
        if need + self.reserved_size > self.cache_manager.available_size:
            self.cache_manager.unlock(handle)
            return None
        row = self.table_manager.allocate()
        return handle, row, np.asarray(handle.get_matched_indices(), dtype=np.int32)

    def _make(self, p: Waiting, handle, row: int, cached_len: int, slots: np.ndarray) -> Req:
        remain = p.prompt_len - cached_len
        chunk = min(self.token_budget, remain)
        cls = ChunkedReq if chunk < remain else Req
        self.token_budget -= chunk
        # Reserve what the request may still allocate: its unprefilled prompt, its outputs and one
        # partial page. Every scheduling step builds a new adder whose base reservation covers only
        # running decode requests, so a continuing chunk is reserved again here, or requests
        # admitted behind it could take the pages its later chunks need.
        self.reserved_size += remain + p.budget + self.cache_manager.page_size - 1
        req = cls(
            input_ids=p.input_ids[: cached_len + chunk],
            table_idx=row,
            cached_len=cached_len,
            output_len=p.budget,
            uid=p.uid,
            sampling_params=p.sampling_params,
            cache_handle=handle,
        )
        req.slots = slots
        # a fresh admission with a cache hit must publish the matched slots to its page-table row
        req.pending_prefix = cached_len if p.chunk is None else 0
        return req

    def try_add_one(self, p: Waiting) -> Req | None:
        if self.token_budget <= 0:
            return None
        if (c := p.chunk) is not None:
            return self._make(p, c.cache_handle, c.table_idx, c.cached_len, c.slots)
        got = self._admit(p)
        if got is None:
            return None
        handle, row, slots = got
        return self._make(p, handle, row, handle.cached_len, slots)


@dataclass
class PrefillManager:
    cache_manager: CacheManager
    table_manager: TableManager
    decode_manager: DecodeManager
    pending_list: List[Waiting] = field(default_factory=list)

    def add_one_req(self, msg) -> None:
        self.pending_list.append(Waiting(msg.uid, msg.input_ids, msg.sampling_params))

    def schedule_next_batch(self, prefill_budget: int) -> Batch | None:
        if not self.pending_list:
            return None
        adder = PrefillAdder(
            token_budget=prefill_budget,
            reserved_size=self.decode_manager.inflight_tokens,
            cache_manager=self.cache_manager,
            table_manager=self.table_manager,
        )
        reqs: List[Req] = []
        chunked: List[Waiting] = []
        for p in self.pending_list:
            r = adder.try_add_one(p)
            if r is None:
                break
            p.chunk = r if isinstance(r, ChunkedReq) else None
            if p.chunk is not None:
                chunked.append(p)
            reqs.append(r)
        if not reqs:
            return None
        self.pending_list = chunked + self.pending_list[len(reqs) :]
        return Batch(reqs=reqs, phase="prefill")

    def abort_req(self, uid: int) -> Req | None:
        for i, p in enumerate(self.pending_list):
            if p.uid == uid:
                self.pending_list.pop(i)
                return p.chunk
        return None

    @property
    def runnable(self) -> bool:
        return bool(self.pending_list)
