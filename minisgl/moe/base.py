from __future__ import annotations

from abc import ABC, abstractmethod

import torch


class BaseMoeBackend(ABC):
    @abstractmethod
    def forward(self, hidden_states: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor,
                gating_output: torch.Tensor, topk: int, renormalize: bool, activation: str = "silu",
                *, w1_bias: torch.Tensor | None = None, w2_bias: torch.Tensor | None = None,
                softmax_after_topk: bool = False, expert_offset: int = 0,
                w1_interleaved: bool = False) -> torch.Tensor: ...
