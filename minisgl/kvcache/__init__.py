"""KV pool + prefix caches (reference: python/minisgl/kvcache/__init__.py:27-62)."""

from __future__ import annotations

from typing import TYPE_CHECKING, Callable

from minisgl.utils import Registry

from .base import (
    BaseCacheHandle,
    BaseKVCachePool,
    BasePrefixCache,
    InsertResult,
    MatchResult,
    SizeInfo,
)

if TYPE_CHECKING:
    import torch

    from minisgl.models import ModelConfig

SUPPORTED_CACHE_MANAGER: Registry[Callable[..., BasePrefixCache]] = Registry("Cache Manager")


@SUPPORTED_CACHE_MANAGER.register("naive")
def _naive(page_size: int = 1) -> BasePrefixCache:
    from .naive_cache import NaivePrefixCache

    return NaivePrefixCache(page_size)


@SUPPORTED_CACHE_MANAGER.register("radix")
def _radix(page_size: int = 1) -> BasePrefixCache:
    from .radix_cache import RadixPrefixCache

    return RadixPrefixCache(page_size)


def create_prefix_cache(type: str, page_size: int = 1) -> BasePrefixCache:
    return SUPPORTED_CACHE_MANAGER[type](page_size)


def create_kvcache_pool(
    model_config: "ModelConfig",
    num_pages: int,
    page_size: int,
    dtype: "torch.dtype",
    device: "torch.device",
) -> BaseKVCachePool:
    from .mha_pool import MHAKVCache

    return MHAKVCache(
        num_kv_heads=model_config.num_kv_heads,
        num_layers=model_config.num_layers,
        head_dim=model_config.head_dim,
        num_pages=num_pages,
        page_size=page_size,
        dtype=dtype,
        device=device,
    )


__all__ = [
    "create_kvcache_pool",
    "create_prefix_cache",
    "BaseKVCachePool",
    "BaseCacheHandle",
    "BasePrefixCache",
    "InsertResult",
    "MatchResult",
    "SizeInfo",
    "SUPPORTED_CACHE_MANAGER",
]
