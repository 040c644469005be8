"""Mixture-of-experts layer (reference: python/minisgl/layers/moe.py:9-59).

Expert weights are packed: ``gate_up_proj [E, 2*I/tp, H]`` as ``[gate; up]`` halves and
``down_proj [E, H, I/tp]``. Two ways to spread them over the tensor-parallel ranks
(``MINISGL_MOE_PARALLEL``):

* ``tp`` (the reference's): every rank holds a 1/tp slice of every expert's intermediate dim;
* ``ep`` (expert parallelism, not in the reference): rank r holds experts
  [r E/tp, (r+1) E/tp) whole, ``[E/tp, 2I, H]``. Attention is tensor-parallel, so every rank
  already has every token's activations: a rank runs the tokens routed to its own experts and
  the all-reduce that follows the layer sums the ranks' contributions (the combine). Each
  expert's GEMMs keep their full intermediate size instead of 1/tp of it.

Either way the sum over ranks follows the expert combine.
"""

from __future__ import annotations

import torch

from minisgl.core import get_global_ctx
from minisgl.parallel import DistributedCommunicator, get_tp_info
from minisgl.utils import div_even

from .base import BaseOP


def moe_parallel_mode() -> str:
    from minisgl.env import ENV

    mode = str(ENV.MOE_PARALLEL).lower()
    if mode not in ("tp", "ep"):
        raise ValueError(f"MINISGL_MOE_PARALLEL must be tp or ep, got {mode!r}")
    return mode


def expert_range(num_experts: int) -> tuple:
    """(first expert, number of experts) this rank holds."""
    info = get_tp_info()
    if info.size == 1 or moe_parallel_mode() == "tp":
        return 0, num_experts
    local = div_even(num_experts, info.size)
    return info.rank * local, local


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
        self._e0, local = expert_range(num_experts)
        self._ep = info.size > 1 and local < num_experts
        inter = intermediate_size if self._ep else div_even(intermediate_size, info.size)
        # shape / dtype placeholders (no memory: the loaded tensors replace them)
        self.gate_up_proj = torch.empty(local, 2 * inter, hidden_size, device="meta")
        self.down_proj = torch.empty(local, hidden_size, inter, device="meta")
        self.gate_up_proj_bias = torch.empty(local, 2 * inter) if has_bias else None
        self.down_proj_bias = torch.empty(local, hidden_size) if has_bias else None
        self._comm = DistributedCommunicator()

    # set by the model when the next norm can take the unreduced per-rank sum (fused all-reduce +
    # RMSNorm); `deferred` tells whether the last forward left it unreduced
    defer_to_norm = False
    deferred = False
    _interleaved = False  # gate_up_proj in the gated grouped-GEMM layout (CUDA)

    def load_state_dict(self, state_dict, *, prefix: str = "", _internal: bool = False) -> None:
        from minisgl.moe.mxfp4 import Mxfp4Experts, dequant_mxfp4, interleave_rows, pad_k

        # MXFP4 experts (``<proj>_blocks`` / ``<proj>_scales``, see models/weight.py): kept in fp4
        # on the GPU for the fp4 grouped GEMM, dequantised elsewhere
        key = (lambda n: f"{prefix}.{n}") if prefix else (lambda n: n)
        fp4 = {}
        for proj in ("gate_up_proj", "down_proj"):
            if key(f"{proj}_blocks") in state_dict:
                blocks, scales = state_dict.pop(key(f"{proj}_blocks")), state_dict.pop(key(f"{proj}_scales"))
                if blocks.is_cuda:
                    fp4[proj] = (blocks, scales)
                    setattr(self, proj, None)  # not a tensor: the state-dict walk skips it
                else:
                    state_dict[key(proj)] = dequant_mxfp4(blocks, scales, getattr(self, proj).dtype)
        super().load_state_dict(state_dict, prefix=prefix, _internal=_internal)
        if not fp4 and not self.gate_up_proj.is_cuda:
            return
        # GPU layout: gate / up rows interleaved in 128-row blocks (intermediate size padded to a
        # whole block) so the first grouped GEMM applies the activation in its epilogue
        from minisgl.ops.moe import interleave_experts

        if "gate_up_proj" in fp4:
            blocks, scales = fp4["gate_up_proj"]
            self.gate_up_proj = Mxfp4Experts.pack(interleave_rows(blocks), interleave_rows(scales), 256)
            if self.gate_up_proj_bias is not None:
                self.gate_up_proj_bias = interleave_rows(self.gate_up_proj_bias)
            ip = self.gate_up_proj.n // 2
            if "down_proj" in fp4:
                blocks, scales = fp4["down_proj"]
                self.down_proj = Mxfp4Experts.pack(*pad_k(blocks, scales, ip), 128)
            elif self.down_proj.shape[2] != ip:
                w2 = torch.zeros(*self.down_proj.shape[:2], ip, dtype=self.down_proj.dtype, device=self.down_proj.device)
                w2[:, :, : self.down_proj.shape[2]] = self.down_proj
                self.down_proj = w2
        else:
            self.gate_up_proj, self.down_proj, self.gate_up_proj_bias = interleave_experts(
                self.gate_up_proj, self.down_proj, self.gate_up_proj_bias)
        self._interleaved = True

    def forward(self, hidden_states: torch.Tensor, router_logits: torch.Tensor) -> torch.Tensor:
        be = get_global_ctx().moe_backend
        out = be.forward(
            hidden_states, self.gate_up_proj, self.down_proj, router_logits, self._top_k,
            self._renorm, self._act, w1_bias=self.gate_up_proj_bias,
            # TP: every rank holds a slice of each expert, so only rank 0 adds the output bias;
            # EP: each expert's output is computed on one rank, which adds its bias
            w2_bias=self.down_proj_bias if (self._tp == 1 or self._ep or get_tp_info().rank == 0) else None,
            softmax_after_topk=self._softmax_after_topk, expert_offset=self._e0,
            w1_interleaved=self._interleaved,
        )
        self.deferred = False
        if self._tp > 1:
            fused = DistributedCommunicator.norm_impl
            if self.defer_to_norm and fused is not None and fused.fits(out):
                self.deferred = True
            else:
                out = self._comm.all_reduce(out)
        return out
