"""Torch helpers: default-dtype context and NVTX ranges
(reference: python/minisgl/utils/torch_utils.py:11-37)."""

from __future__ import annotations

import functools
from contextlib import contextmanager

import torch


@contextmanager
def torch_dtype(dtype: torch.dtype):
    old = torch.get_default_dtype()
    torch.set_default_dtype(dtype)
    try:
        yield
    finally:
        torch.set_default_dtype(old)


def nvtx_annotate(name: str, layer_id_field: str | None = None):
    """Wrap a method in an NVTX range (for Nsight traces) when ``MINISGL_NVTX=1``. ``name`` may
    contain ``{}``, filled from ``getattr(self, layer_id_field)``. The ranges land in eager runs
    and in CUDA-graph captures (reference: python/minisgl/utils/torch_utils.py:23-37)."""
    from minisgl.env import ENV

    def deco(fn):
        @functools.wraps(fn)
        def inner(*args, **kwargs):
            if not ENV.NVTX or not torch.cuda.is_available():
                return fn(*args, **kwargs)
            label = name.format(getattr(args[0], layer_id_field)) if layer_id_field else name
            torch.cuda.nvtx.range_push(label)
            try:
                return fn(*args, **kwargs)
            finally:
                torch.cuda.nvtx.range_pop()

        return inner

    return deco
