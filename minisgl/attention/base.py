"""Attention backend interface (reference: python/minisgl/attention/base.py:18-63)."""

from __future__ import annotations

from abc import ABC, abstractmethod
from typing import TYPE_CHECKING, List

import torch

if TYPE_CHECKING:
    from minisgl.core import Batch


class BaseAttnMetadata(ABC):
    @abstractmethod
    def get_last_indices(self, bs: int) -> torch.Tensor: ...


class BaseAttnBackend(ABC):
    @abstractmethod
    def forward(self, q: torch.Tensor, layer_id: int, batch: "Batch", *, window: int = -1,
                sinks: torch.Tensor | None = None) -> torch.Tensor: ...

    @abstractmethod
    def prepare_metadata(self, batch: "Batch", host: dict) -> None: ...

    def init_capture_graph(self, max_seq_len: int, bs_list: List[int]) -> None:
        raise NotImplementedError

    def prepare_for_capture(self, batch: "Batch") -> None:
        raise NotImplementedError

    def prepare_for_replay(self, batch: "Batch") -> None:
        raise NotImplementedError
