"""Abstract interfaces of the KV pool and the prefix caches
(reference: python/minisgl/kvcache/base.py:10-135).

Slot indices handed out by a prefix cache are *host* int32 numpy arrays in this engine: all
allocator and tree bookkeeping stays on the CPU and reaches the GPU as one packed copy per batch.
"""

from __future__ import annotations

from abc import ABC, abstractmethod
from dataclasses import dataclass
from typing import NamedTuple

import numpy as np
import torch


class BaseKVCachePool(ABC):
    @abstractmethod
    def k_cache(self, layer_id: int) -> torch.Tensor: ...

    @abstractmethod
    def v_cache(self, layer_id: int) -> torch.Tensor: ...

    @abstractmethod
    def store_kv(self, k: torch.Tensor, v: torch.Tensor, out_loc: torch.Tensor, layer_id: int) -> None: ...

    @property
    @abstractmethod
    def device(self) -> torch.device: ...

    @property
    @abstractmethod
    def dtype(self) -> torch.dtype: ...

    @property
    @abstractmethod
    def num_layers(self) -> int: ...


@dataclass(frozen=True)
class BaseCacheHandle(ABC):
    cached_len: int

    @abstractmethod
    def get_matched_indices(self) -> np.ndarray: ...


class SizeInfo(NamedTuple):
    evictable_size: int
    protected_size: int

    @property
    def total_size(self) -> int:
        return self.evictable_size + self.protected_size


class InsertResult(NamedTuple):
    cached_len: int  # length that was already cached (the caller frees its duplicate slots)
    handle: BaseCacheHandle


class MatchResult(NamedTuple):
    cuda_handle: BaseCacheHandle


class BasePrefixCache(ABC):
    @abstractmethod
    def lock_handle(self, handle: BaseCacheHandle, unlock: bool = False) -> None:
        """Pin (or unpin) the matched path so eviction cannot take it."""

    @abstractmethod
    def match_prefix(self, input_ids: torch.Tensor) -> MatchResult:
        """Longest cached page-aligned prefix of ``input_ids``."""

    @abstractmethod
    def insert_prefix(self, input_ids: torch.Tensor, indices) -> InsertResult:
        """Insert the page-aligned prefix with its KV slot indices."""

    @abstractmethod
    def evict(self, size: int) -> np.ndarray:
        """Evict at least ``size`` tokens of unreferenced entries; returns the freed slots."""

    @abstractmethod
    def reset(self) -> None: ...

    @property
    @abstractmethod
    def size_info(self) -> SizeInfo: ...

    @abstractmethod
    def check_integrity(self) -> None: ...


def as_host_int32(x) -> np.ndarray:
    if isinstance(x, torch.Tensor):
        x = x.detach().to("cpu", torch.int32).numpy()
    return np.ascontiguousarray(x, dtype=np.int32)
