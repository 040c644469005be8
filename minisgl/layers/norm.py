"""RMSNorm layers (reference: python/minisgl/layers/norm.py:8-38)."""

from __future__ import annotations

from typing import Tuple

import torch

from minisgl import ops

from .base import BaseOP


class RMSNorm(BaseOP):
    def __init__(self, size: int, eps: float):
        self.weight = torch.empty(size)
        self._eps = eps

    @property
    def eps(self) -> float:
        return self._eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.rmsnorm(x, self.weight, self._eps)


class RMSNormFused(RMSNorm):
    """``(x, residual) -> (norm(x + residual), x + residual)``; the first layer passes
    ``residual=None`` and gets ``(norm(x), x)``."""

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None) -> Tuple[torch.Tensor, torch.Tensor]:
        if residual is None:
            return ops.rmsnorm(x, self.weight, self._eps), x
        return ops.fused_add_rmsnorm(x, residual, self.weight, self._eps)

    def forward_unreduced(self, x: torch.Tensor, residual: torch.Tensor | None) -> Tuple[torch.Tensor, torch.Tensor]:
        """``x`` is this rank's partial sum of a row-parallel linear: all-reduce it, add the
        residual and normalise, in one fused collective kernel."""
        from minisgl.parallel.comm import DistributedCommunicator

        return DistributedCommunicator.norm_impl.all_reduce_add_rmsnorm(x, residual, self.weight, self._eps)
