"""Routed-expert forward on the GPU (graph-capturable, no host synchronization):

route (softmax top-k) -> align (counting sort into per-expert segments padded to ``bn`` rows,
device work list) -> gather permuted activations -> grouped tcgen05 GEMM (gate|up, activation in
its epilogue when the weights are gate/up interleaved) -> grouped GEMM (down) -> weighted top-k
combine. Expert weights are bf16 ``[E, N, K]`` tensors or MXFP4 ``Mxfp4Experts`` (fp4 in HBM,
converted to bf16 tile by tile inside the grouped GEMM).

Behaviour matches ``moe/grouped.py:moe_reference`` (and the reference's fused MoE,
python/minisgl/moe/fused.py:127-227).
"""

from __future__ import annotations

import torch

from minisgl._native import cuda as _cuda

_ACT = {"silu": 0, "gelu": 1, "swiglu_oai": 2}
_GATED_EPI = {"silu": 1, "gelu": 2, "swiglu_oai": 4}  # grouped-GEMM epilogue applying the activation


def interleave_experts(w1: torch.Tensor, w2: torch.Tensor, b1: torch.Tensor | None = None):
    """Expert weights for the gated grouped GEMM: ``w1 [E, 2I, H]`` as [gate; up] halves -> gate / up
    rows interleaved in blocks of GATE_UP_BLOCK (one 256-row weight tile then holds 128 gate rows and
    their 128 up rows, and the epilogue applies the activation). I is padded up to a whole block with
    zero rows (and ``w2 [E, H, I]`` with zero columns, ``b1`` with zeros): act(0, 0) * ... = 0 for
    SiLU, GELU and the clamped SwiGLU alike, so padding contributes nothing. Returns (w1, w2, b1)."""
    from .reference import GATE_UP_BLOCK

    E, two_i, H = w1.shape
    inter = two_i // 2
    ip = -(-inter // GATE_UP_BLOCK) * GATE_UP_BLOCK
    nb = ip // GATE_UP_BLOCK
    w1n = torch.zeros(E, 2 * ip, H, dtype=w1.dtype, device=w1.device)
    v = w1n.view(E, nb, 2, GATE_UP_BLOCK, H)  # [expert, block, gate/up, row, H]
    for half in range(2):
        src = torch.zeros(E, ip, H, dtype=w1.dtype, device=w1.device) if ip != inter else None
        part = w1[:, half * inter : (half + 1) * inter]
        if src is not None:
            src[:, :inter] = part
            part = src
        v[:, :, half] = part.reshape(E, nb, GATE_UP_BLOCK, H)
    w2n = w2
    if ip != inter:
        w2n = torch.zeros(E, w2.shape[1], ip, dtype=w2.dtype, device=w2.device)
        w2n[:, :, :inter] = w2
    b1n = None
    if b1 is not None:
        b1n = torch.zeros(E, 2 * ip, dtype=b1.dtype, device=b1.device)
        vb = b1n.view(E, nb, 2, GATE_UP_BLOCK)
        for half in range(2):
            part = torch.zeros(E, ip, dtype=b1.dtype, device=b1.device)
            part[:, :inter] = b1[:, half * inter : (half + 1) * inter]
            vb[:, :, half] = part.view(E, nb, GATE_UP_BLOCK)
    return w1n, w2n, b1n


def pick_bn(pairs: int, experts: int) -> int:
    avg = pairs / max(experts, 1)
    for bn in (16, 32, 64):
        if avg <= bn:
            return bn
    return 128


def _grouped(out, xs, w, bias, count, work, bn, epi):
    """Grouped GEMM over bf16 experts ``[E, N, K]`` or MXFP4 experts kept in fp4 (``Mxfp4Experts``)."""
    from minisgl.moe.mxfp4 import Mxfp4Experts

    if isinstance(w, Mxfp4Experts):
        _cuda().gemm_grouped_fp4(out, xs, w.q, w.s, w.n, bias, count, work, bn, epi)
    else:
        _cuda().gemm_grouped(out, xs, w, bias, count, work, bn, epi)


def moe_forward(x, w1, w2, gating, topk, renormalize, activation, w1_bias=None, w2_bias=None,
                softmax_after_topk=False, expert_offset: int = 0, w1_interleaved: bool = False):
    """``w1``/``w2`` hold experts [expert_offset, expert_offset + E) of the ``gating`` columns
    (expert parallelism); assignments to other experts contribute nothing here. With
    ``w1_interleaved`` (``interleave_experts`` layout) the first grouped GEMM's epilogue applies the
    activation; otherwise a separate kernel does."""
    c = _cuda()
    T, H = x.shape
    E, two_i, _ = w1.shape
    inter = two_i // 2
    dev = x.device
    logits = gating if gating.dtype == torch.float32 else gating.float()
    weights = torch.empty(T, topk, dtype=torch.float32, device=dev)
    ids = torch.empty(T, topk, dtype=torch.int32, device=dev)
    c.moe_route(logits.contiguous(), topk, bool(renormalize), bool(softmax_after_topk), weights, ids)
    pairs = T * topk
    bn = pick_bn(pairs, E)
    max_tiles = (pairs + bn - 1) // bn + E
    rows = max_tiles * bn
    perm = torch.empty(rows, dtype=torch.int32, device=dev)
    inv = torch.empty(pairs, dtype=torch.int32, device=dev)
    work = torch.empty(max_tiles, 2, dtype=torch.int32, device=dev)
    count = torch.empty(1, dtype=torch.int32, device=dev)
    c.moe_align(ids, E, bn, perm, inv, work, count, expert_offset)
    xs = torch.empty(rows, H, dtype=x.dtype, device=dev)
    c.moe_gather(xs, x.contiguous(), perm, topk)
    a = torch.empty(rows, inter, dtype=x.dtype, device=dev)
    if w1_interleaved:
        _grouped(a, xs, w1, w1_bias, count, work, bn, _GATED_EPI[activation])
    else:
        y1 = torch.empty(rows, two_i, dtype=x.dtype, device=dev)
        _grouped(y1, xs, w1, w1_bias, count, work, bn, 0)
        c.moe_act(a, y1, _ACT[activation], perm)
    y2 = torch.empty(rows, H, dtype=x.dtype, device=dev)
    _grouped(y2, a, w2, w2_bias, count, work, bn, 0)
    out = torch.empty(T, H, dtype=x.dtype, device=dev)
    c.moe_combine(out, y2, weights, inv, topk)
    return out
