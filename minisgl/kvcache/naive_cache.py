"""Prefix cache that never reuses anything (reference: python/minisgl/kvcache/naive_cache.py)."""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .base import BaseCacheHandle, BasePrefixCache, InsertResult, MatchResult, SizeInfo

_EMPTY = np.empty(0, dtype=np.int32)


@dataclass(frozen=True)
class NaiveCacheHandle(BaseCacheHandle):
    def get_matched_indices(self) -> np.ndarray:
        return _EMPTY


class NaivePrefixCache(BasePrefixCache):
    def __init__(self, page_size: int = 1):
        self.page_size = page_size

    def lock_handle(self, handle, unlock: bool = False) -> None:
        pass

    def match_prefix(self, input_ids) -> MatchResult:
        return MatchResult(NaiveCacheHandle(0))

    def insert_prefix(self, input_ids, indices) -> InsertResult:
        return InsertResult(0, NaiveCacheHandle(0))

    def evict(self, size: int) -> np.ndarray:
        if size == 0:
            return _EMPTY
        raise RuntimeError("naive prefix cache holds nothing to evict")

    def reset(self) -> None:
        pass

    @property
    def size_info(self) -> SizeInfo:
        return SizeInfo(0, 0)

    def check_integrity(self) -> None:
        pass
