"""MoE backends. One implementation (this engine's kernels); ``fused``/``auto`` are accepted
names (reference: python/minisgl/moe/__init__.py:19-27)."""

from __future__ import annotations

from minisgl.utils import Registry

from .base import BaseMoeBackend
from .grouped import GroupedMoe

SUPPORTED_MOE_BACKENDS: Registry = Registry("MoE Backend")
for _n in ("auto", "fused", "grouped"):
    SUPPORTED_MOE_BACKENDS.register(_n)(GroupedMoe)


def create_moe_backend(name: str = "auto") -> BaseMoeBackend:
    return SUPPORTED_MOE_BACKENDS[name]()


__all__ = ["BaseMoeBackend", "GroupedMoe", "create_moe_backend", "SUPPORTED_MOE_BACKENDS"]
