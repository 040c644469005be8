"""Tensor-parallel linear layers (reference: python/minisgl/layers/linear.py:13-127).

Weights are ``[out, in]`` bf16 (nn.Linear layout), i.e. K-major for the sm_100a GEMM, which puts
the weight rows in the MMA's M slot (swap-AB) so a decode batch of any size fills the N slot.
"""

from __future__ import annotations

from typing import List

import torch

from minisgl import ops
from minisgl.parallel import DistributedCommunicator, get_tp_info
from minisgl.utils import div_even

from .base import BaseOP


class _Linear(BaseOP):
    def __init__(self, in_features: int, out_features: int, has_bias: bool):
        self.weight = torch.empty(out_features, in_features)
        self.bias = torch.empty(out_features) if has_bias else None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.linear(x, self.weight, self.bias)


class LinearReplicated(_Linear):
    def __init__(self, in_features: int, out_features: int, has_bias: bool = False):
        super().__init__(in_features, out_features, has_bias)


class LinearColParallelMerged(_Linear):
    """Several column-parallel projections stacked along the output dim (e.g. gate+up)."""

    def __init__(self, in_features: int, out_sizes: List[int], has_bias: bool = False):
        tp = get_tp_info().size
        self.local_sizes = [div_even(s, tp) for s in out_sizes]
        super().__init__(in_features, sum(self.local_sizes), has_bias)


class LinearQKVMerged(_Linear):
    def __init__(self, hidden_size: int, head_dim: int, num_qo_heads: int, num_kv_heads: int, has_bias: bool = False):
        tp = get_tp_info().size
        self.local_q = div_even(num_qo_heads, tp)
        self.local_kv = div_even(num_kv_heads, tp, allow_replicate=True)
        super().__init__(hidden_size, (self.local_q + 2 * self.local_kv) * head_dim, has_bias)


class LinearRowParallel(_Linear):
    """Input-split linear followed by a sum over TP ranks."""

    def __init__(self, in_features: int, out_features: int, has_bias: bool = False, reduce: bool = True):
        info = get_tp_info()
        self._tp = info.size
        self._reduce = reduce
        self._comm = DistributedCommunicator()
        # set by blocks whose next op is an RMSNorm that can take the unreduced partial sum (the
        # norm then runs the fused all-reduce + residual add + RMSNorm); `deferred` tells the block
        # whether the last forward did so
        self.defer_to_norm = False
        self.deferred = False
        super().__init__(div_even(in_features, info.size), out_features, has_bias)
        if has_bias and info.rank != 0:
            self._bias_scale = 0.0  # only rank 0 adds the bias before the sum
        else:
            self._bias_scale = 1.0

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        bias = self.bias if (self.bias is not None and self._bias_scale) else None
        self.deferred = False
        fused = DistributedCommunicator.norm_impl if (self._tp > 1 and self._reduce and self.defer_to_norm) else None
        if fused is not None and x.is_cuda:
            # GEMM fused with the collective: the output tiles land in this rank's NVLS staging
            # region and the GEMM signals the other ranks itself (None: batch too small or too large)
            y = fused.linear_into_staging(x, self.weight, bias)
            if y is not None:
                self.deferred = True
                return y
        y = ops.linear(x, self.weight, bias)
        if self._tp > 1 and self._reduce:
            if fused is not None and fused.fits(y):
                self.deferred = True
            else:
                y = self._comm.all_reduce(y)
        return y


class LinearOProj(LinearRowParallel):
    pass
