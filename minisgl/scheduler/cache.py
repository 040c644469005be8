"""Page allocator + prefix cache glue (reference: python/minisgl/scheduler/cache.py:15-146).

All state is host-side: the free list is a numpy array of page-start slots, and the token-level
page table mirror needed for caching lives in each request's ``slots`` array. Page-table updates
for the device are emitted as (row, pos, slot) triples that the batch plan uploads in one copy.
"""

from __future__ import annotations

from contextlib import contextmanager
from typing import List, Tuple

import numpy as np

from minisgl.core import Req
from minisgl.kvcache import BaseCacheHandle, MatchResult, create_prefix_cache
from minisgl.utils import div_ceil


class CacheManager:
    def __init__(self, num_pages: int, page_size: int, cache_type: str):
        self.num_pages = num_pages
        self.page_size = page_size
        self.free_pages = np.arange(num_pages, dtype=np.int32) * page_size
        self.prefix_cache = create_prefix_cache(cache_type, page_size)
        self._lazy: List[np.ndarray] | None = None

    # ---------------------------------------------------------------- admission helpers
    def match_req(self, input_ids) -> MatchResult:
        if len(input_ids) == 0:
            raise ValueError("empty prompt")
        # keep >= 1 token to compute so the request produces logits
        return self.prefix_cache.match_prefix(input_ids[: len(input_ids) - 1])

    @property
    def available_size(self) -> int:
        return self.prefix_cache.size_info.evictable_size + len(self.free_pages) * self.page_size

    def lock(self, handle: BaseCacheHandle) -> None:
        self.prefix_cache.lock_handle(handle, unlock=False)

    def unlock(self, handle: BaseCacheHandle) -> None:
        self.prefix_cache.lock_handle(handle, unlock=True)

    # ---------------------------------------------------------------- allocation
    def allocate_paged(self, reqs: List[Req]) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
        """Give every request slots for ``[cached_len, device_len)``. Returns page-table writes
        ``(rows, positions, slots)`` for the device copy, and extends each ``req.slots``."""
        ps = self.page_size
        spans = []
        need = 0
        rows, poss, slots = [], [], []
        for r in reqs:
            n = r.pending_prefix
            if n:
                rows.append(np.full(n, r.table_idx, dtype=np.int32))
                poss.append(np.arange(n, dtype=np.int32))
                slots.append(r.slots[:n])
                r.pending_prefix = 0
            c, d = r.cached_len, r.device_len
            if d - c == 1:  # decode: a new page only when the token starts one
                if c % ps == 0:
                    spans.append((r, c // ps, c // ps + 1))
                    need += 1
                continue
            first, last = div_ceil(c, ps), div_ceil(d, ps)
            if last > first:
                spans.append((r, first, last))
                need += last - first
        if need == 0 and not rows:
            e = np.empty(0, dtype=np.int32)
            return e, e, e
        pages = self._allocate(need) if need else np.empty(0, np.int32)
        offs = np.arange(ps, dtype=np.int32)
        k = 0
        for r, first, last in spans:
            n = last - first
            tok = (pages[k : k + n, None] + offs[None, :]).reshape(-1)
            k += n
            r.slots = np.concatenate([r.slots[: first * ps], tok])
            rows.append(np.full(n * ps, r.table_idx, dtype=np.int32))
            poss.append(np.arange(first * ps, last * ps, dtype=np.int32))
            slots.append(tok)
        return np.concatenate(rows), np.concatenate(poss), np.concatenate(slots)

    def _allocate(self, n: int) -> np.ndarray:
        free = len(self.free_pages)
        if n > free:
            evicted = self.prefix_cache.evict((n - free) * self.page_size)
            self.free_pages = np.concatenate([self.free_pages, evicted[:: self.page_size]])
            if len(self.free_pages) < n:
                raise RuntimeError("KV pool exhausted after eviction")
        out, self.free_pages = self.free_pages[:n], self.free_pages[n:]
        return out

    def _free(self, slots: np.ndarray) -> None:
        if len(slots) == 0:
            return
        pages = slots[:: self.page_size]
        if self._lazy is not None:
            self._lazy.append(pages)
        else:
            self.free_pages = np.concatenate([self.free_pages, pages])

    @contextmanager
    def lazy_free_region(self):
        """Batch all frees inside the region into one concatenate."""
        self._lazy = []
        try:
            yield
        finally:
            parts, self._lazy = self._lazy, None
            if parts:
                self.free_pages = np.concatenate([self.free_pages] + parts)

    # ---------------------------------------------------------------- caching
    def cache_req(self, req: Req, *, finished: bool) -> None:
        """Insert the computed prefix of ``req`` into the prefix cache and free what became
        redundant. Slot ranges (all within ``req.slots``):

        * ``[0, old.cached_len)`` was matched from the cache at admission;
        * ``[old.cached_len, prefix)`` was computed by this request but meanwhile cached by
          another one: free ours;
        * ``[prefix, new.cached_len)`` is now owned by the cache;
        * ``[new.cached_len, cached_len)`` is the unaligned tail: free it if finished.
        """
        ids = req.input_ids[: req.cached_len]
        slots = req.slots[: req.cached_len]
        old = req.cache_handle
        prefix, new = self.prefix_cache.insert_prefix(ids, slots)
        self.unlock(old)
        self._free(slots[old.cached_len : prefix])
        if finished:
            self._free(slots[new.cached_len :])
        else:
            if prefix > old.cached_len:
                # The pages just freed were this request's own copy of a prefix that another
                # request cached first. The request keeps decoding, so its page-table row must
                # point at the cached copy before its next forward, or it would read pages that
                # are about to be handed out again (the reference keeps its own page indices
                # here: python/minisgl/scheduler/cache.py:70-79).
                cached = np.asarray(new.get_matched_indices()[old.cached_len : prefix], dtype=np.int32)
                req.slots = req.slots.copy()
                req.slots[old.cached_len : prefix] = cached
                req.pending_prefix = max(req.pending_prefix, prefix)
            req.cache_handle = new
            self.lock(new)

    def check_integrity(self) -> None:
        self.prefix_cache.check_integrity()
        cached_pages = self.prefix_cache.size_info.total_size // self.page_size
        if len(self.free_pages) + cached_pages != self.num_pages:
            raise RuntimeError(
                f"cache integrity: free({len(self.free_pages)}) + cached({cached_pages}) "
                f"!= total({self.num_pages})"
            )
        if len(np.unique(self.free_pages)) != len(self.free_pages):
            raise RuntimeError("cache integrity: duplicate free pages")
        if self.page_size > 1 and np.any(self.free_pages % self.page_size):
            raise RuntimeError("cache integrity: unaligned free page")
