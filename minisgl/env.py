"""Typed ``MINISGL_*`` environment flags, parsed once at import.

Same variable names and defaults as the reference (python/minisgl/env.py:58-87) plus the
flags this engine adds for its native paths (fused collectives, timeouts).
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Any, Callable


def _as_bool(text: str) -> bool:
    return text.strip().lower() in ("1", "true", "yes", "on")


def _as_opt_bool(text: str) -> bool | None:
    t = text.strip().lower()
    if t in ("", "none", "auto"):
        return None
    return _as_bool(t)


def parse_mem_bytes(text: str) -> int:
    """Parse ``"1G"``, ``"512M"``, ``"64KB"`` or a plain integer into bytes."""
    t = text.strip().upper()
    if t.endswith("B") and len(t) > 1 and t[-2].isalpha():
        t = t[:-1]
    units = {"K": 1 << 10, "M": 1 << 20, "G": 1 << 30, "T": 1 << 40}
    if t and t[-1] in units:
        return int(float(t[:-1]) * units[t[-1]])
    return int(t)


@dataclass
class _Flag:
    default: Any
    parse: Callable[[str], Any]


_FLAGS = {
    # interactive shell sampling defaults
    "SHELL_MAX_TOKENS": _Flag(2048, int),
    "SHELL_TOP_K": _Flag(-1, int),
    "SHELL_TOP_P": _Flag(1.0, float),
    "SHELL_TEMPERATURE": _Flag(0.6, float),
    # runtime
    "FLASHINFER_USE_TENSOR_CORES": _Flag(None, _as_opt_bool),  # accepted, unused (own kernels)
    "DISABLE_OVERLAP_SCHEDULING": _Flag(False, _as_bool),
    "PYNCCL_MAX_BUFFER_SIZE": _Flag(1 << 30, parse_mem_bytes),
    # engine-specific
    "COMM_MODE": _Flag("auto", str),  # auto | nccl | fused
    "COMM_TIMEOUT_MS": _Flag(5000, int),  # bound on every device-side peer wait
    "DEBUG_CHECK_INTEGRITY": _Flag(False, _as_bool),
    "NVTX": _Flag(False, _as_bool),  # NVTX ranges around layers / attention / MLP / LM head / sampler
    "MOE_PARALLEL": _Flag("tp", str),  # tp: shard every expert's intermediate dim; ep: whole experts per rank
    "BOUNDS_CHECK": _Flag(False, _as_bool),  # load the index-checking kernel build (_cuda_bc)
    "NVLS_LL_BYTES": _Flag(2 << 20, parse_mem_bytes),  # largest world x T x H x 4 sent in the LL form
    "NVLS_GEMM_FUSION": _Flag(True, _as_bool),  # row-parallel GEMMs write the NVLS staging region
    "FUSED_LM_HEAD": _Flag(True, _as_bool),  # greedy batches take the argmax in the LM-head GEMM epilogue
    "MXFP4_RESIDENT": _Flag(True, _as_bool),  # keep MXFP4 experts in fp4 on the GPU (fp4 grouped GEMM)
}


class _Env:
    """Attribute access to the parsed flags: ``ENV.DISABLE_OVERLAP_SCHEDULING``."""

    PREFIX = "MINISGL_"

    def __init__(self) -> None:
        self.reload()

    def reload(self) -> None:
        for name, flag in _FLAGS.items():
            raw = os.environ.get(self.PREFIX + name)
            value = flag.default
            if raw is not None:
                try:
                    value = flag.parse(raw)
                except (TypeError, ValueError):
                    value = flag.default
            object.__setattr__(self, name, value)

    def __setattr__(self, key: str, value: Any) -> None:  # tests may override flags
        if key not in _FLAGS:
            raise AttributeError(key)
        object.__setattr__(self, key, value)


ENV = _Env()

__all__ = ["ENV", "parse_mem_bytes"]
