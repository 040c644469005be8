"""Routed-expert forward on the GPU (graph-capturable, no host synchronization):

route (softmax top-k) -> align (counting sort into per-expert segments padded to ``bn`` rows,
device work list) -> gather permuted activations -> grouped tcgen05 GEMM (gate|up) -> activation
-> grouped GEMM (down) -> weighted top-k combine.

Behaviour matches ``moe/grouped.py:moe_reference`` (and the reference's fused MoE,
python/minisgl/moe/fused.py:127-227).
"""

from __future__ import annotations

import torch

from minisgl._native import cuda as _cuda

_ACT = {"silu": 0, "gelu": 1, "swiglu_oai": 2}


def pick_bn(pairs: int, experts: int) -> int:
    avg = pairs / max(experts, 1)
    for bn in (16, 32, 64):
        if avg <= bn:
            return bn
    return 128


def moe_forward(x, w1, w2, gating, topk, renormalize, activation, w1_bias=None, w2_bias=None,
                softmax_after_topk=False, expert_offset: int = 0):
    """``w1``/``w2`` hold experts [expert_offset, expert_offset + E) of the ``gating`` columns
    (expert parallelism); assignments to other experts contribute nothing here."""
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
    y1 = torch.empty(rows, two_i, dtype=x.dtype, device=dev)
    c.gemm_grouped(y1, xs, w1, w1_bias, count, work, bn)
    a = torch.empty(rows, inter, dtype=x.dtype, device=dev)
    c.moe_act(a, y1, _ACT[activation], perm)
    y2 = torch.empty(rows, H, dtype=x.dtype, device=dev)
    c.gemm_grouped(y2, a, w2, w2_bias, count, work, bn)
    out = torch.empty(T, H, dtype=x.dtype, device=dev)
    c.moe_combine(out, y2, weights, inv, topk)
    return out
