"""Op entry points used by the layers.

CUDA tensors run this engine's sm_100a kernels (``minisgl._cuda``); CPU tensors run the PyTorch
reference in ``ops.reference`` (the oracle / CPU engine). There is no third path: on a GPU a
missing extension raises instead of falling back.
"""

from __future__ import annotations

import torch

from minisgl._native import cuda as _cuda

from . import reference as ref
from .reference import GATE_UP_BLOCK, deinterleave_gate_up, interleave_gate_up


def _on_gpu(t: torch.Tensor) -> bool:
    return t.is_cuda


def embedding(weight, ids, vocab_start: int = 0, vocab_len: int | None = None):
    if not _on_gpu(weight):
        return ref.embedding(weight, ids, vocab_start, vocab_len)
    out = torch.empty(ids.shape[0], weight.shape[1], dtype=weight.dtype, device=weight.device)
    lo, n = (0, weight.shape[0]) if vocab_len is None else (vocab_start, vocab_len)
    _cuda().embedding(out, weight, ids, lo, n, vocab_len is not None)
    return out


def rmsnorm(x, w, eps: float):
    if not _on_gpu(x):
        return ref.rmsnorm(x, w, eps)
    out = torch.empty_like(x)
    _cuda().rmsnorm(out, x, w, eps)
    return out


def fused_add_rmsnorm(x, residual, w, eps: float):
    if not _on_gpu(x):
        return ref.fused_add_rmsnorm(x, residual, w, eps)
    _cuda().fused_add_rmsnorm(x, residual, w, eps)
    return x, residual


def linear(x, w, bias=None):
    if not _on_gpu(x):
        return ref.linear(x, w, bias)
    out = torch.empty(x.shape[0], w.shape[0], dtype=x.dtype, device=x.device)
    _cuda().gemm(out, x, w, bias, 0)
    return out


def linear_f32(x, w, bias=None):
    """``x @ w^T (+ bias)`` with fp32 output (the MoE router: expert selection compares logits
    that bf16 rounding would often tie)."""
    if not _on_gpu(x):
        return ref.linear(x.float(), w.float(), None if bias is None else bias.float())
    out = torch.empty(x.shape[0], w.shape[0], dtype=torch.float32, device=x.device)
    _cuda().gemm(out, x, w, bias, 3)
    return out


def lm_head_argmax(x, w, bias, n_valid: int, id_offset: int = 0):
    """(id_offset + argmax over the first ``n_valid`` rows of ``x @ w^T (+ bias)``, its value) per
    row of ``x``; on the GPU the argmax runs in the GEMM epilogue and no logits are written. Ties
    resolve to the lowest id."""
    if not _on_gpu(x):
        logits = ref.linear(x, w[:n_valid], None if bias is None else bias[:n_valid]).float()
        vals, idx = logits.max(dim=-1)
        return idx.to(torch.int32) + id_offset, vals
    ids = torch.empty(x.shape[0], dtype=torch.int32, device=x.device)
    vals = torch.empty(x.shape[0], dtype=torch.float32, device=x.device)
    _cuda().lm_head_argmax(ids, vals, x.contiguous(), w, bias, n_valid, id_offset)
    return ids, vals


def gate_up_silu(x, w, act: str = "silu"):
    if not _on_gpu(x):
        return ref.gate_up_silu(x, w, act)
    out = torch.empty(x.shape[0], w.shape[0] // 2, dtype=x.dtype, device=x.device)
    _cuda().gemm(out, x, w, None, 1 if act == "silu" else 2)
    return out


def silu_and_mul(x):
    if not _on_gpu(x):
        return ref.silu_and_mul(x)
    out = torch.empty(x.shape[0], x.shape[1] // 2, dtype=x.dtype, device=x.device)
    _cuda().act_and_mul(out, x, 0)
    return out


def gelu_and_mul(x):
    if not _on_gpu(x):
        return ref.gelu_and_mul(x)
    out = torch.empty(x.shape[0], x.shape[1] // 2, dtype=x.dtype, device=x.device)
    _cuda().act_and_mul(out, x, 1)
    return out


def qk_norm_rope_store(qkv, positions, cos_sin, q_norm, k_norm, eps, k_cache, v_cache, out_loc, nq, nkv, hd):
    if not _on_gpu(qkv):
        return ref.qk_norm_rope_store(
            qkv, positions, cos_sin, q_norm, k_norm, eps, k_cache, v_cache, out_loc, nq, nkv, hd
        )
    q = torch.empty(qkv.shape[0], nq, hd, dtype=qkv.dtype, device=qkv.device)
    _cuda().qk_norm_rope_store(
        q, qkv, positions, cos_sin, q_norm, k_norm, eps, k_cache, v_cache, out_loc, nq, nkv, hd
    )
    return q


def store_kv(k, v, k_cache, v_cache, out_loc):
    if not _on_gpu(k):
        return ref.store_kv(k, v, k_cache, v_cache, out_loc)
    _cuda().store_kv(k.reshape(k.shape[0], -1), v.reshape(v.shape[0], -1), k_cache, v_cache, out_loc)


def argmax(logits, vocab: int | None = None, with_values: bool = False):
    """Row argmax over the first ``vocab`` columns (all by default); ties to the lowest index.
    ``with_values`` also returns each row's maximum (fp32)."""
    if not _on_gpu(logits):
        lf = logits[:, :vocab].float() if vocab is not None else logits.float()
        vals, idx = lf.max(dim=-1)  # first maximal index
        idx = idx.to(torch.int32)
        return (idx, vals) if with_values else idx
    out = torch.empty(logits.shape[0], dtype=torch.int32, device=logits.device)
    vals = torch.empty(logits.shape[0], dtype=torch.float32, device=logits.device) if with_values else None
    _cuda().argmax(out, logits, vals, -1 if vocab is None else vocab)
    return (out, vals) if with_values else out


def sample(logits, temperature, top_k, top_p, seed, step, col_ids=None, id_offset: int = 0,
           with_values: bool = False):
    """Temperature / top-k / top-p draw per row. Column j is token ``col_ids[row, j]`` (a
    candidate list sorted by id) or ``id_offset + j`` (a vocabulary shard); token ids are returned.
    ``with_values`` also returns each row's winning score, for combining shards."""
    if not _on_gpu(logits):
        return ref.sample(logits, temperature, top_k, top_p, seed, step, col_ids, id_offset, with_values)
    out = torch.empty(logits.shape[0], dtype=torch.int32, device=logits.device)
    vals = torch.empty(logits.shape[0], dtype=torch.float32, device=logits.device) if with_values else None
    _cuda().sample(out, logits, temperature, top_k, top_p, seed, step, col_ids, id_offset, vals)
    return (out, vals) if with_values else out


__all__ = [
    "GATE_UP_BLOCK",
    "interleave_gate_up",
    "deinterleave_gate_up",
    "embedding",
    "rmsnorm",
    "fused_add_rmsnorm",
    "linear",
    "linear_f32",
    "lm_head_argmax",
    "gate_up_silu",
    "silu_and_mul",
    "gelu_and_mul",
    "qk_norm_rope_store",
    "store_kv",
    "argmax",
    "sample",
    "ref",
]
