"""Attention backends. This engine has one implementation (its own sm_100a kernels); the
reference's backend names (``fa``, ``fi``, ``trtllm``, ``"p,d"`` hybrids, ``auto``) are accepted on the
command line and all resolve to it (reference registry: python/minisgl/attention/__init__.py:19-68)."""

from __future__ import annotations

from minisgl.utils import Registry

from .base import BaseAttnBackend, BaseAttnMetadata
from .paged import PagedAttentionBackend, PagedMetadata

SUPPORTED_ATTENTION_BACKENDS: Registry = Registry("Attention Backend")
for _name in ("auto", "paged", "fa", "fi", "trtllm"):
    SUPPORTED_ATTENTION_BACKENDS.register(_name)(PagedAttentionBackend)


def validate_attn_backend(name: str) -> str:
    for part in name.split(","):
        SUPPORTED_ATTENTION_BACKENDS.assert_supported(part.strip())
    return name


def create_attention_backend(name: str, model_config, device) -> BaseAttnBackend:
    validate_attn_backend(name)
    return PagedAttentionBackend(
        model_config.num_qo_heads, model_config.num_kv_heads, model_config.head_dim, device
    )


__all__ = [
    "BaseAttnBackend",
    "BaseAttnMetadata",
    "PagedAttentionBackend",
    "PagedMetadata",
    "create_attention_backend",
    "validate_attn_backend",
    "SUPPORTED_ATTENTION_BACKENDS",
]
