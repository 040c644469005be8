"""Loaders for the in-tree native extensions.

``host()`` returns the host C++ runtime (radix tree); it is rebuilt on demand because it only
needs a C++ compiler. ``cuda()`` returns the sm_100a kernel library and raises if it was not built:
a GPU run never silently falls back to PyTorch.
"""

from __future__ import annotations

import functools
import importlib


@functools.cache
def host():
    try:
        return importlib.import_module("minisgl._host")
    except ImportError:
        from minisgl import _build

        _build.build_host()
        return importlib.import_module("minisgl._host")


@functools.cache
def cuda():
    try:
        import torch  # noqa: F401  (loads libtorch before the extension)

        return importlib.import_module("minisgl._cuda")
    except ImportError as e:
        raise RuntimeError(
            "minisgl CUDA kernels are not built; run `python -m minisgl._build` "
            f"(or __graft_entry__.build()) first: {e}"
        ) from e
