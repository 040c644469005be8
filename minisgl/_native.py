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


class _CountingModule:
    """Forwards attribute access to the extension and counts kernel-launching calls."""

    _NON_LAUNCH = {"get_error", "num_sms", "gemm_splits", "peer_flag_bytes", "peer_alloc", "peer_free",
                   "ipc_handle", "ipc_open", "ipc_close", "peer_grid", "nvls_grid", "nvls_flag_bytes",
                   "nvls_state_words", "nvls_ticket_offset", "gemm_force_bn", "attention_prefill_trace"}

    def __init__(self, mod):
        self._mod = mod

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        if name in self._NON_LAUNCH or not callable(fn):
            return fn
        from minisgl.engine.counters import COUNTERS

        def call(*args, **kwargs):
            COUNTERS.launches += 2 if (name == "attention_decode" and args[-2] > 1) else 1
            return fn(*args, **kwargs)

        return call


@functools.cache
def cuda():
    try:
        import torch  # noqa: F401  (loads libtorch before the extension)

        from minisgl.env import ENV

        name = "minisgl._cuda_bc" if ENV.BOUNDS_CHECK else "minisgl._cuda"
        return _CountingModule(importlib.import_module(name))
    except ImportError as e:
        raise RuntimeError(
            "minisgl CUDA kernels are not built; run `python -m minisgl._build` "
            f"(or __graft_entry__.build()) first: {e}"
        ) from e
