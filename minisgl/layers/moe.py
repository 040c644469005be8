"""Mixture-of-experts layer (reference: python/minisgl/layers/moe.py:9-59).

Expert weights are packed: ``gate_up_proj [E, 2*I/tp, H]`` as ``[gate; up]`` halves and
``down_proj [E, H, I/tp]``. Tensor parallelism shards every
expert's intermediate dim; the sum over ranks follows the expert combine.
"""

from __future__ import annotations

import torch

from minisgl.core import get_global_ctx
from minisgl.parallel import DistributedCommunicator, get_tp_info
from minisgl.utils import div_even

from .base import BaseOP


class MoELayer(BaseOP):
    def __init__(self, num_experts: int, top_k: int, hidden_size: int, intermediate_size: int,
                 renormalize: bool = True, activation: str = "silu", has_bias: bool = False,
                 routing: str = "softmax_topk"):
        info = get_tp_info()
        self._tp = info.size
        self._top_k = top_k
        self._renorm = renormalize
        self._act = activation
        self._num_experts = num_experts
        self._softmax_after_topk = routing == "topk_softmax"
        inter = div_even(intermediate_size, info.size)
        self.gate_up_proj = torch.empty(num_experts, 2 * inter, hidden_size)
        self.down_proj = torch.empty(num_experts, hidden_size, inter)
        self.gate_up_proj_bias = torch.empty(num_experts, 2 * inter) if has_bias else None
        self.down_proj_bias = torch.empty(num_experts, hidden_size) if has_bias else None
        self._comm = DistributedCommunicator()

    def forward(self, hidden_states: torch.Tensor, router_logits: torch.Tensor) -> torch.Tensor:
        be = get_global_ctx().moe_backend
        out = be.forward(
            hidden_states, self.gate_up_proj, self.down_proj, router_logits, self._top_k,
            self._renorm, self._act, w1_bias=self.gate_up_proj_bias,
            w2_bias=self.down_proj_bias if (self._tp == 1 or get_tp_info().rank == 0) else None,
            softmax_after_topk=self._softmax_after_topk,
        )
        if self._tp > 1:
            out = self._comm.all_reduce(out)
        return out
