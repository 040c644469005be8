"""Device capability checks (reference: python/minisgl/utils/arch.py:7-29)."""

from __future__ import annotations

import functools

import torch


@functools.cache
def _cap() -> tuple[int, int]:
    if not torch.cuda.is_available():
        return (0, 0)
    return torch.cuda.get_device_capability()


def is_sm90_supported() -> bool:
    return _cap() == (9, 0)


def is_sm100_supported() -> bool:
    return _cap()[0] == 10
