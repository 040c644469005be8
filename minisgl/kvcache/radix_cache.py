"""Radix prefix cache backed by the C++ tree in ``csrc/host/radix_tree.cpp``
(reference behaviour: python/minisgl/kvcache/radix_cache.py:101-237)."""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from minisgl._native import host

from .base import (
    BaseCacheHandle,
    BasePrefixCache,
    InsertResult,
    MatchResult,
    SizeInfo,
    as_host_int32,
)


@dataclass(frozen=True)
class RadixCacheHandle(BaseCacheHandle):
    node: int = field(default=0)
    tree: object = field(default=None, repr=False, compare=False)

    def get_matched_indices(self) -> np.ndarray:
        return self.tree.indices(self.node)


class RadixPrefixCache(BasePrefixCache):
    def __init__(self, page_size: int = 1):
        self.page_size = page_size
        self.tree = host().RadixTree(page_size)

    def lock_handle(self, handle: BaseCacheHandle, unlock: bool = False) -> None:
        assert isinstance(handle, RadixCacheHandle)
        if unlock:
            self.tree.unlock(handle.node)
        else:
            self.tree.lock(handle.node)

    def match_prefix(self, input_ids) -> MatchResult:
        node, length = self.tree.match(as_host_int32(input_ids))
        return MatchResult(RadixCacheHandle(int(length), node, self.tree))

    def insert_prefix(self, input_ids, indices) -> InsertResult:
        prefix, node = self.tree.insert(as_host_int32(input_ids), as_host_int32(indices))
        n = len(input_ids) - len(input_ids) % self.page_size
        return InsertResult(int(prefix), RadixCacheHandle(n, node, self.tree))

    def evict(self, size: int) -> np.ndarray:
        return self.tree.evict(int(size))

    def reset(self) -> None:
        if self.tree.protected_size:
            raise RuntimeError("cannot reset a radix cache with locked entries")
        self.tree = host().RadixTree(self.page_size)

    @property
    def size_info(self) -> SizeInfo:
        return SizeInfo(self.tree.evictable_size, self.tree.protected_size)

    def check_integrity(self) -> None:
        self.tree.check_integrity()
