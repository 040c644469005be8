"""Routed-expert execution: softmax top-k routing, token sort by expert, grouped GEMMs with a
gated activation between them, then the weighted top-k combine
(reference flow: python/minisgl/moe/fused.py:9-256)."""

from __future__ import annotations

import torch
import torch.nn.functional as F

from minisgl.ops import reference as ref

from .base import BaseMoeBackend


def route(gating: torch.Tensor, topk: int, renormalize: bool, softmax_after_topk: bool = False):
    """Returns (weights fp32 [T, k], ids int32 [T, k])."""
    g = gating.float()
    if softmax_after_topk:  # gpt-oss: top-k on logits, softmax over the selected k
        vals, ids = torch.topk(g, topk, dim=-1)
        return torch.softmax(vals, dim=-1), ids.to(torch.int32)
    p = torch.softmax(g, dim=-1)
    w, ids = torch.topk(p, topk, dim=-1)
    if renormalize:
        w = w / w.sum(-1, keepdim=True)
    return w, ids.to(torch.int32)


def expert_act(y: torch.Tensor, activation: str) -> torch.Tensor:
    """Expert gate_up output [T, 2I] laid out as [gate | up] halves -> activated [T, I]."""
    g, u = y.float().chunk(2, dim=-1)
    if activation == "silu":
        a = F.silu(g) * u
    elif activation == "gelu":
        a = F.gelu(g, approximate="tanh") * u
    elif activation == "swiglu_oai":  # gpt-oss: clamped, alpha=1.702, (up + 1)
        g = g.clamp(max=7.0)
        u = u.clamp(-7.0, 7.0)
        a = (g * torch.sigmoid(1.702 * g)) * (u + 1)
    else:
        raise ValueError(activation)
    return a


def moe_reference(x, w1, w2, gating, topk, renormalize, activation, w1_bias=None, w2_bias=None,
                  softmax_after_topk=False, expert_offset: int = 0):
    """``w1``/``w2`` hold experts [expert_offset, expert_offset + E) (expert parallelism)."""
    w, ids = route(gating, topk, renormalize, softmax_after_topk)
    out = torch.zeros(x.shape[0], w2.shape[1], dtype=torch.float32, device=x.device)
    xf = x.float()
    E = w1.shape[0]
    for e in torch.unique(ids).tolist():
        le = e - expert_offset
        if not 0 <= le < E:
            continue
        tok, slot = torch.nonzero(ids == e, as_tuple=True)
        y = xf[tok] @ w1[le].float().t()
        if w1_bias is not None:
            y = y + w1_bias[le].float()
        a = expert_act(y, activation)
        z = a @ w2[le].float().t()
        if w2_bias is not None:
            z = z + w2_bias[le].float()
        out.index_add_(0, tok, z * w[tok, slot, None])
    return out.to(x.dtype)


class GroupedMoe(BaseMoeBackend):
    def forward(self, hidden_states, w1, w2, gating_output, topk, renormalize, activation="silu",
                *, w1_bias=None, w2_bias=None, softmax_after_topk=False, expert_offset=0, w1_interleaved=False):
        if not hidden_states.is_cuda:
            return moe_reference(hidden_states, w1, w2, gating_output, topk, renormalize, activation,
                                 w1_bias, w2_bias, softmax_after_topk, expert_offset)
        from minisgl.ops.moe import moe_forward

        return moe_forward(hidden_states, w1, w2, gating_output, topk, renormalize, activation,
                           w1_bias, w2_bias, softmax_after_topk, expert_offset, w1_interleaved)
