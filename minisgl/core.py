"""Core request/batch state shared by the scheduler and the engine
(reference: python/minisgl/core.py:15-136).

A ``Req`` tracks three lengths over one page-table row:
``cached_len`` tokens already have KV in the pool, ``device_len`` tokens are known on the device
(prompt plus generated so far), and ``max_device_len`` is the hard cap (prompt + max_tokens).
Each forward computes KV for ``[cached_len, device_len)`` and samples the token at ``device_len``.
"""

from __future__ import annotations

from contextlib import contextmanager
from dataclasses import dataclass, field
from typing import TYPE_CHECKING, Any, List, Literal

import torch

if TYPE_CHECKING:
    from minisgl.attention import BaseAttnBackend, BaseAttnMetadata
    from minisgl.kvcache import BaseCacheHandle, BaseKVCachePool
    from minisgl.moe import BaseMoeBackend


# max_tokens of a request without a limit of its own: the scheduler clamps it to the context left
UNBOUNDED_MAX_TOKENS = 1 << 30


@dataclass
class SamplingParams:
    temperature: float = 0.0
    top_k: int = -1
    top_p: float = 1.0
    ignore_eos: bool = False
    max_tokens: int = 1024
    seed: int | None = None  # per-request RNG seed (None: derived from the request uid)

    @property
    def is_greedy(self) -> bool:
        return (self.temperature <= 0.0 or self.top_k == 1) and self.top_p >= 1.0


class Req:
    """One running request. ``input_ids`` (CPU int32, prompt + tokens sampled so far) is a view
    of a buffer sized for the whole request, so appending a sampled token is an in-place write."""

    def __init__(self, input_ids: torch.Tensor, table_idx: int, cached_len: int, output_len: int,
                 uid: int, sampling_params: SamplingParams, cache_handle: "BaseCacheHandle") -> None:
        if input_ids.device.type != "cpu":
            raise ValueError("Req.input_ids must live on the CPU")
        self.table_idx = table_idx
        self.cached_len = cached_len
        self.output_len = output_len
        self.uid = uid
        self.sampling_params = sampling_params
        self.cache_handle = cache_handle
        self.greedy = sampling_params.is_greedy
        self.pending_prefix = 0  # matched prefix slots still to be written into the page table
        self.aborted = False  # resources released on abort; results of in-flight batches are dropped
        n = len(input_ids)
        self.device_len = n
        self.max_device_len = n + output_len
        if not (0 <= cached_len < n <= self.max_device_len):
            raise ValueError(f"bad lengths for {self!r}")
        self._buf = torch.empty(self.max_device_len + 1, dtype=torch.int32)
        self._buf[:n] = input_ids
        self._np = self._buf.numpy()
        self._len = n

    @property
    def input_ids(self) -> torch.Tensor:
        return self._buf[: self._len]

    @property
    def host_len(self) -> int:
        """Tokens known on the host. Under overlap scheduling ``device_len`` runs one step ahead
        (the next batch is launched before this one's tokens are read back)."""
        return self._len

    @property
    def remain_len(self) -> int:
        return self.max_device_len - self.device_len

    @property
    def extend_len(self) -> int:
        return self.device_len - self.cached_len

    def complete_one(self) -> None:
        """Advance after a forward was launched: the KV of the extend part now exists and one
        more token (being sampled) will exist on the device."""
        self.cached_len = self.device_len
        self.device_len += 1

    def append_host(self, next_token: int) -> None:
        self._np[self._len] = next_token
        self._len += 1

    @property
    def can_decode(self) -> bool:
        return self.remain_len > 0

    def __repr__(self) -> str:
        return (
            f"{type(self).__name__}(uid={self.uid}, table_idx={self.table_idx}, "
            f"cached_len={self.cached_len}, device_len={getattr(self, 'device_len', '?')}, "
            f"max_device_len={getattr(self, 'max_device_len', '?')})"
        )


@dataclass
class Batch:
    reqs: List[Req]
    phase: Literal["prefill", "decode"]
    # filled by the scheduler
    input_ids: torch.Tensor = field(init=False)
    positions: torch.Tensor = field(init=False)
    out_loc: torch.Tensor = field(init=False)
    padded_reqs: List[Req] = field(init=False)
    # filled by the attention backend
    attn_metadata: "BaseAttnMetadata" = field(init=False)

    @property
    def is_prefill(self) -> bool:
        return self.phase == "prefill"

    @property
    def is_decode(self) -> bool:
        return self.phase == "decode"

    @property
    def size(self) -> int:
        return len(self.reqs)

    @property
    def padded_size(self) -> int:
        return len(self.padded_reqs)


@dataclass
class Context:
    """Process-global handles the layers read during a forward."""

    page_size: int
    page_table: torch.Tensor = field(init=False)  # [rows, max_len] int32 token slots
    attn_backend: "BaseAttnBackend" = field(init=False)
    moe_backend: "BaseMoeBackend" = field(init=False)
    kv_cache: "BaseKVCachePool" = field(init=False)
    extras: dict = field(default_factory=dict)
    _batch: Batch | None = field(default=None, init=False)

    @property
    def batch(self) -> Batch:
        if self._batch is None:
            raise RuntimeError("no active batch in context")
        return self._batch

    @contextmanager
    def forward_batch(self, batch: Batch):
        if self._batch is not None:
            raise RuntimeError("nested forward_batch")
        self._batch = batch
        try:
            yield
        finally:
            self._batch = None


_GLOBAL_CTX: Context | None = None


def set_global_ctx(ctx: Context) -> None:
    global _GLOBAL_CTX
    if _GLOBAL_CTX is not None:
        raise RuntimeError("global context already set")
    _GLOBAL_CTX = ctx


def get_global_ctx() -> Context:
    if _GLOBAL_CTX is None:
        raise RuntimeError("global context not set")
    return _GLOBAL_CTX


def reset_global_ctx(ctx: Any = None) -> Context | None:
    """Swap the global context (tests, engine shutdown). Returns the previous one."""
    global _GLOBAL_CTX
    old, _GLOBAL_CTX = _GLOBAL_CTX, ctx
    return old
