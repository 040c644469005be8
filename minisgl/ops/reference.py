"""Plain PyTorch (fp32-accumulating) implementations of every op.

They are the numerics oracle for the CUDA kernels and the execution path of the CPU engine
(the tiny-model and gloo tensor-parallel tests). They define the exact semantics each kernel in
``csrc/kernels`` must reproduce.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

GATE_UP_BLOCK = 128  # gate/up rows are interleaved in blocks of this many rows


def embedding(weight: torch.Tensor, ids: torch.Tensor, vocab_start: int = 0, vocab_len: int | None = None):
    ids = ids.long()
    if vocab_len is None:
        return weight[ids]
    local = ids - vocab_start
    mask = (local >= 0) & (local < vocab_len)
    out = weight[local.clamp(0, weight.shape[0] - 1)]
    return out * mask.unsqueeze(-1).to(out.dtype)


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (y * w.float()).to(x.dtype)


def fused_add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float):
    """residual <- x + residual ; x <- rmsnorm(residual). In place, returns (x, residual)."""
    s = x.float() + residual.float()
    residual.copy_(s.to(residual.dtype))
    x.copy_(rmsnorm(residual, w, eps))
    return x, residual


def linear(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    y = x.float() @ w.float().t()
    if bias is not None:
        y = y + bias.float()
    return y.to(x.dtype)


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """[I, H] gate and up -> [2I, H] with blocks of GATE_UP_BLOCK rows alternating g/u."""
    i, h = gate.shape
    b = GATE_UP_BLOCK
    assert i % b == 0, f"intermediate size {i} must be a multiple of {b}"
    return torch.stack([gate.view(i // b, b, h), up.view(i // b, b, h)], dim=1).reshape(2 * i, h)


def deinterleave_gate_up(y: torch.Tensor):
    t, n2 = y.shape
    b = GATE_UP_BLOCK
    v = y.view(t, n2 // (2 * b), 2, b)
    return v[:, :, 0].reshape(t, -1), v[:, :, 1].reshape(t, -1)


def gate_up_act(y: torch.Tensor, act: str = "silu") -> torch.Tensor:
    """Activation over an interleaved gate/up projection output [T, 2I] -> [T, I]."""
    g, u = deinterleave_gate_up(y.float())
    a = F.silu(g) if act == "silu" else F.gelu(g, approximate="tanh")
    return (a * u).to(y.dtype)


def gate_up_silu(x: torch.Tensor, w: torch.Tensor, act: str = "silu") -> torch.Tensor:
    g, u = deinterleave_gate_up(x.float() @ w.float().t())
    a = F.silu(g) if act == "silu" else F.gelu(g, approximate="tanh")
    return (a * u).to(x.dtype)


def silu_and_mul(x: torch.Tensor) -> torch.Tensor:
    g, u = x.float().chunk(2, dim=-1)
    return (F.silu(g) * u).to(x.dtype)


def gelu_and_mul(x: torch.Tensor) -> torch.Tensor:
    g, u = x.float().chunk(2, dim=-1)
    return (F.gelu(g, approximate="tanh") * u).to(x.dtype)


def rope(x: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor) -> torch.Tensor:
    """Neox-style rotary on [T, heads, hd] with cos_sin[pos] = [cos(hd/2) | sin(hd/2)]."""
    hd = x.shape[-1]
    cs = cos_sin[positions.long()].float()
    cos, sin = cs[:, None, : hd // 2], cs[:, None, hd // 2 :]
    x1, x2 = x.float()[..., : hd // 2], x.float()[..., hd // 2 :]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1).to(x.dtype)


def qk_norm_rope_store(
    qkv: torch.Tensor,
    positions: torch.Tensor,
    cos_sin: torch.Tensor,
    q_norm: torch.Tensor | None,
    k_norm: torch.Tensor | None,
    eps: float,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    out_loc: torch.Tensor,
    nq: int,
    nkv: int,
    hd: int,
) -> torch.Tensor:
    """Split qkv [T, (nq+2nkv)*hd]; per-head RMSNorm on q/k (if weights given); RoPE on q/k;
    store k/v rows at ``out_loc``; return q [T, nq, hd]."""
    t = qkv.shape[0]
    q = qkv[:, : nq * hd].reshape(t, nq, hd)
    k = qkv[:, nq * hd : (nq + nkv) * hd].reshape(t, nkv, hd)
    v = qkv[:, (nq + nkv) * hd :].reshape(t, nkv, hd)
    if q_norm is not None:
        q = rmsnorm(q, q_norm, eps)
        k = rmsnorm(k, k_norm, eps)
    q = rope(q, positions, cos_sin)
    k = rope(k, positions, cos_sin)
    store_kv(k, v, k_cache, v_cache, out_loc)
    return q.contiguous()


def store_kv(k, v, k_cache, v_cache, out_loc) -> None:
    idx = out_loc.long()
    k_cache.view(k_cache.shape[0], -1)[idx] = k.reshape(k.shape[0], -1).to(k_cache.dtype)
    v_cache.view(v_cache.shape[0], -1)[idx] = v.reshape(v.shape[0], -1).to(v_cache.dtype)


def paged_attention(
    q: torch.Tensor,  # [T, nq, hd]
    k_cache: torch.Tensor,  # [slots, nkv, hd]
    v_cache: torch.Tensor,
    page_table: torch.Tensor,  # [rows, L] int32 slot per position
    rows: torch.Tensor,  # [B]
    cu_q: torch.Tensor,  # [B+1]
    kv_lens: torch.Tensor,  # [B]
    sm_scale: float,
    window: int = -1,  # keys with pos <= qpos - window are masked (sliding window), -1 = off
    sinks: torch.Tensor | None = None,  # [nq] learned per-head sink logits
) -> torch.Tensor:
    """Causal attention over the paged cache. Query i of request b sits at position
    ``kv_len[b] - q_len[b] + i``."""
    nq, hd = q.shape[1], q.shape[2]
    nkv = k_cache.shape[1]
    g = nq // nkv
    out = torch.empty_like(q)
    cu = cu_q.tolist()
    lens = kv_lens.tolist()
    rws = rows.tolist()
    for b in range(len(lens)):
        s, e = cu[b], cu[b + 1]
        if e == s:
            continue
        L = lens[b]
        slots = page_table[rws[b], :L].long()
        k = k_cache[slots].float()  # [L, nkv, hd]
        v = v_cache[slots].float()
        qb = q[s:e].float()  # [n, nq, hd]
        n = e - s
        kx = k.repeat_interleave(g, dim=1)
        vx = v.repeat_interleave(g, dim=1)
        scores = torch.einsum("qhd,khd->hqk", qb, kx) * sm_scale
        qpos = torch.arange(L - n, L, device=q.device)[:, None]
        kpos = torch.arange(L, device=q.device)[None, :]
        mask = kpos <= qpos
        if window > 0:
            mask &= kpos > qpos - window
        scores = scores.masked_fill(~mask[None], float("-inf"))
        if sinks is not None:
            sk = sinks.float()[:, None, None].expand(nq, n, 1)
            p = torch.softmax(torch.cat([scores, sk], dim=-1), dim=-1)[..., :-1]
        else:
            p = torch.softmax(scores, dim=-1)
        out[s:e] = torch.einsum("hqk,khd->qhd", p, vx).to(q.dtype)
    return out


def argmax(logits: torch.Tensor) -> torch.Tensor:
    return torch.argmax(logits.float(), dim=-1).to(torch.int32)


def _uniform_from_counter(seed: torch.Tensor, step: torch.Tensor, vocab: int,
                          ids: torch.Tensor | None = None) -> torch.Tensor:
    """Counter-based uniforms in (0,1) keyed by (seed, step, token id); same hash as the kernel.
    Token ids are ``ids`` ([rows, vocab]) when given, else 0..vocab-1."""
    M = 0xFFFFFFFF
    idx = torch.arange(vocab, dtype=torch.int64)[None, :] if ids is None else ids.long()
    x = (seed.long()[:, None] * 0x9E3779B1 + step.long()[:, None] * 0x85EBCA77 + idx * 0xC2B2AE3D) & M
    for _ in range(2):  # murmur3 finalizer rounds
        x ^= x >> 16
        x = (x * 0x85EBCA6B) & M
        x ^= x >> 13
        x = (x * 0xC2B2AE35) & M
        x ^= x >> 16
    return ((x >> 8).double() + 0.5) / float(1 << 24)


def sample(
    logits: torch.Tensor,
    temperature: torch.Tensor,
    top_k: torch.Tensor,
    top_p: torch.Tensor,
    seed: torch.Tensor,
    step: torch.Tensor,
    col_ids: torch.Tensor | None = None,
    id_offset: int = 0,
    with_values: bool = False,
):
    """Temperature / top-k / top-p sampling by the Gumbel-max trick with counter-based noise:
    keep tokens inside the top-k and the top-p nucleus of softmax(logits / T), then return
    argmax(logits / T - log(-log(u))). Rows with temperature <= 0 are greedy.

    Column j of a row is token ``col_ids[row, j]`` (a candidate list in ascending id order) or
    ``id_offset + j`` (a vocabulary shard); the noise is keyed by the token id and the token id is
    returned. ``with_values`` also returns the winning score (the maximum logit on greedy rows)."""
    lf = logits.float()
    bs, V = lf.shape
    pos = torch.empty(bs, dtype=torch.int64)
    vals = torch.empty(bs, dtype=torch.float32)
    ids = col_ids.cpu() if col_ids is not None else None
    u = _uniform_from_counter(seed.cpu(), step.cpu(), V,
                              None if ids is None and id_offset == 0 else
                              (ids if ids is not None else torch.arange(V)[None, :] + id_offset)).to(lf.device)
    if u.shape[0] == 1 and bs > 1:
        u = u.expand(bs, V)
    for i in range(bs):
        t = float(temperature[i])
        if t <= 0:
            pos[i] = int(torch.argmax(lf[i]))
            vals[i] = float(lf[i, pos[i]])
            continue
        z = lf[i] / t
        k = int(top_k[i])
        keep = torch.ones(V, dtype=torch.bool, device=lf.device)
        if 0 < k < V:
            kth = torch.topk(z, k).values[-1]
            keep &= z >= kth
        p = float(top_p[i])
        if p < 1.0:
            probs = torch.softmax(z.masked_fill(~keep, float("-inf")), -1)
            sp, si = torch.sort(probs, descending=True)
            cum = torch.cumsum(sp, 0)
            cut = int(torch.searchsorted(cum, torch.tensor(p, device=cum.device)).item())
            thr = sp[min(cut, V - 1)]
            keep &= probs >= thr
        g = z.double() - torch.log(-torch.log(u[i]))
        g = g.masked_fill(~keep, float("-inf"))
        pos[i] = int(torch.argmax(g))
        vals[i] = float(g[pos[i]])
    if ids is not None:
        out = ids.gather(1, pos.view(bs, 1)).view(bs).to(torch.int32)
    else:
        out = (pos + id_offset).to(torch.int32)
    out = out.to(logits.device)
    return (out, vals.to(logits.device)) if with_values else out


def rope_cos_sin(max_pos: int, rotary_dim: int, inv_freq: torch.Tensor) -> torch.Tensor:
    t = torch.arange(max_pos, dtype=torch.float32)
    f = torch.outer(t, inv_freq.float())
    return torch.cat([f.cos(), f.sin()], dim=-1)


def default_inv_freq(rotary_dim: int, base: float) -> torch.Tensor:
    return 1.0 / (base ** (torch.arange(0, rotary_dim, 2, dtype=torch.float64) / rotary_dim)).float()


def softmax_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)
