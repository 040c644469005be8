"""Streaming safetensors loader with tensor-parallel sharding
(reference: python/minisgl/models/weight.py:16-124).

Per tensor: strip the ``language_model.`` prefix, skip vision weights, take this rank's shard
(q/k/v/gate/up and their biases split on dim 0 with KV-head replication when tp > kv heads;
o/down split on dim 1; embed/lm_head split into ``ceil(V/tp)`` vocab rows, zero padded; sinks
split by head), merge q,k,v -> ``qkv_proj`` and gate,up -> ``gate_up_proj`` (gate/up interleaved
in 128-row blocks for the fused activation epilogue; expert weights keep plain ``[gate; up]``
halves), and stack per-expert tensors into packed
``[E, ...]`` tensors. Yields ``(name, tensor)`` already on the target device.

gpt-oss checkpoints store each MoE layer's experts fused: ``experts.gate_up_proj`` ``[E, H, 2I]``
(gate / up interleaved along the last dim), ``experts.down_proj`` ``[E, I, H]`` and their biases, or
the MXFP4 form ``experts.{gate_up,down}_proj_{blocks,scales}``: e2m1 values two per byte (low
nibble first) in blocks of 32 along the input dim, one e8m0 scale (bias 127) per block. Both are
converted here to this engine's ``[E, rows, K]`` row-major experts with ``[gate; up]`` halves,
dequantising MXFP4 to the model dtype (reference format: transformers' gpt-oss modeling and mxfp4
integration; mini-sglang itself has no gpt-oss).
"""

from __future__ import annotations

import glob
import os
import re
from typing import Dict, Iterator, Tuple

import torch

from minisgl.moe.mxfp4 import dequant_mxfp4  # noqa: F401  (re-exported for checkpoint tools)
from minisgl.ops.reference import GATE_UP_BLOCK, interleave_gate_up
from minisgl.parallel import get_tp_info
from minisgl.utils import div_ceil

_DIM0 = (".q_proj.", ".k_proj.", ".v_proj.", ".gate_proj.", ".up_proj.")
_DIM1 = (".o_proj.weight", ".down_proj.weight")
_QKV = {".q_proj.": "q", ".k_proj.": "k", ".v_proj.": "v"}
_GU = {".gate_proj.": "gate", ".up_proj.": "up"}
_EXPERT = re.compile(r"^(?P<pre>.+\.experts)\.(?P<idx>\d+)\.(?P<name>.+)$")

def _keep_mxfp4() -> bool:
    from minisgl.env import ENV

    return bool(ENV.MXFP4_RESIDENT)


def _split_gate_up_rows(w: torch.Tensor, rank: int, size: int) -> torch.Tensor:
    """``[E, 2I, ...]`` with gate / up rows interleaved -> this rank's ``[E, 2I/tp, ...]`` as
    ``[gate; up]`` halves (``size`` 1: whole experts)."""
    gate, up = w[:, 0::2], w[:, 1::2]
    if size > 1:
        gate, up = gate.chunk(size, dim=1)[rank], up.chunk(size, dim=1)[rank]
    return torch.cat([gate, up], dim=1).contiguous()


def _fused_expert(key: str, t: torch.Tensor, pending: Dict[str, torch.Tensor], rank: int, size: int, dtype,
                  experts: tuple | None = None):
    """Convert one gpt-oss fused-expert tensor; returns ``(name, tensor)``, ``None`` while an MXFP4
    blocks / scales pair is incomplete (a list of two: the pair kept as MXFP4), or ``False`` if
    ``key`` is not such a tensor. With
    ``experts = (first, count)`` (expert parallelism) only those experts are kept, whole."""
    if experts is not None and t.dim() >= 2 and ".experts." in key:
        t = t[experts[0] : experts[0] + experts[1]]
        rank, size = 0, 1
    for proj in ("gate_up_proj", "down_proj"):
        for part in ("_blocks", "_scales"):
            if key.endswith(f".experts.{proj}{part}"):
                base = key[: -len(part)]
                pending[key] = t
                if f"{base}_blocks" not in pending or f"{base}_scales" not in pending:
                    return None
                blocks, scales = pending.pop(f"{base}_blocks"), pending.pop(f"{base}_scales")
                if _keep_mxfp4():
                    # kept as MXFP4 (the MoE layer packs it for the fp4 grouped GEMM): rows permuted
                    # and split as the bf16 weights would be; the down projection's input dim splits
                    # across ranks in whole 32-value blocks only
                    if proj == "gate_up_proj":  # [E, 2I, H/32, 16], rows interleaved
                        return [(f"{base}_blocks", _split_gate_up_rows(blocks, rank, size)),
                                (f"{base}_scales", _split_gate_up_rows(scales, rank, size))]
                    if size == 1 or scales.shape[-1] % size == 0:  # [E, H, I/32, 16]
                        if size > 1:
                            blocks, scales = blocks.chunk(size, dim=2)[rank], scales.chunk(size, dim=2)[rank]
                        return [(f"{base}_blocks", blocks.contiguous()), (f"{base}_scales", scales.contiguous())]
                w = dequant_mxfp4(blocks, scales, dtype)
                if proj == "gate_up_proj":  # [E, 2I, H], rows interleaved
                    return base, _split_gate_up_rows(w, rank, size)
                return base, (w.chunk(size, dim=-1)[rank] if size > 1 else w).contiguous()  # [E, H, I]
    if key.endswith(".experts.gate_up_proj") and t.dim() == 3:  # [E, H, 2I]
        return key, _split_gate_up_rows(t.transpose(1, 2), rank, size)
    if key.endswith(".experts.gate_up_proj_bias") and t.dim() == 2:  # [E, 2I]
        return key, _split_gate_up_rows(t, rank, size)
    if key.endswith(".experts.down_proj") and t.dim() == 3:  # [E, I, H]
        w = t.transpose(1, 2)
        return key, (w.chunk(size, dim=-1)[rank] if size > 1 else w).contiguous()
    if key.endswith(".experts.down_proj_bias") and t.dim() == 2:  # [E, H]: whole on every rank
        return key, t.contiguous()
    return False


def shard_tensor(key: str, t: torch.Tensor, rank: int, size: int, num_kv_heads: int, head_dim: int) -> torch.Tensor:
    if size == 1:
        return t
    if any(s in key for s in _DIM0):
        if (".k_proj." in key or ".v_proj." in key) and num_kv_heads < size:
            h = rank * num_kv_heads // size
            return t[h * head_dim : (h + 1) * head_dim].clone()
        return t.chunk(size, dim=0)[rank].clone()
    if any(key.endswith(s) for s in _DIM1):
        return t.chunk(size, dim=-1)[rank].clone()
    if key.endswith(".sinks"):
        return t.chunk(size, dim=0)[rank].clone()
    if "embed_tokens" in key or "lm_head" in key:
        per = div_ceil(t.shape[0], size)
        part = t[rank * per : min((rank + 1) * per, t.shape[0])]
        if part.shape[0] < per:
            pad = torch.zeros((per - part.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
            part = torch.cat([part, pad])
        return part.clone()
    return t


def _merge_slot(key: str):
    for sub, slot in _QKV.items():
        if sub in key:
            return key.replace(sub, ".qkv_proj."), slot, ("q", "k", "v")
    for sub, slot in _GU.items():
        if sub in key:
            return key.replace(sub, ".gate_up_proj."), slot, ("gate", "up")
    return None


def _pad_to_block(t: torch.Tensor, dim: int) -> torch.Tensor:
    """Zero-pad a dense MLP shard along ``dim`` to a whole number of gate/up interleave blocks
    (the layer sizes come from ``padded_intermediate``)."""
    n = t.shape[dim]
    pad = -n % GATE_UP_BLOCK
    if pad == 0:
        return t
    shape = list(t.shape)
    shape[dim] = pad
    return torch.cat([t, t.new_zeros(shape)], dim=dim)


def _finish_merge(key: str, parts: Dict[str, torch.Tensor]) -> torch.Tensor:
    if "gate_up_proj" in key and ".experts." in key:  # experts keep [gate; up] halves
        return torch.cat([parts["gate"], parts["up"]], dim=0)
    if "gate_up_proj" in key:
        g, u = _pad_to_block(parts["gate"], 0), _pad_to_block(parts["up"], 0)
        if g.dim() == 1:  # bias
            return interleave_gate_up(g[:, None], u[:, None])[:, 0]
        return interleave_gate_up(g, u)
    return torch.cat([parts["q"], parts["k"], parts["v"]], dim=0)


def _expert_key(key: str):
    m = _EXPERT.match(key)
    if m is None:
        return None
    name = m.group("name").removesuffix(".weight")
    if name.endswith(".bias"):  # stacked expert biases are `<proj>_bias` tensors of the MoE layer
        name = name[: -len(".bias")] + "_bias"
    return f"{m.group('pre')}.{name}", int(m.group("idx"))


def load_weight(model_path: str, device: torch.device, config=None) -> Iterator[Tuple[str, torch.Tensor]]:
    import safetensors

    from minisgl.utils.hf import cached_load_hf_config, download_hf_weight

    from .config import ModelConfig

    folder = download_hf_weight(model_path)
    config = config or ModelConfig.from_hf(cached_load_hf_config(model_path))
    files = sorted(glob.glob(os.path.join(folder, "*.safetensors")))
    files = [f for f in files if not f.endswith("consolidated.safetensors")] or files
    if not files:
        raise FileNotFoundError(f"no *.safetensors under {folder}")
    info = get_tp_info()
    merge: Dict[str, Dict[str, torch.Tensor]] = {}
    experts: Dict[str, Dict[int, torch.Tensor]] = {}
    pending: Dict[str, torch.Tensor] = {}  # gpt-oss MXFP4 blocks / scales awaiting their pair
    dtype = getattr(config, "dtype", None) or torch.bfloat16
    ep = None  # expert parallelism: (first expert, count) held by this rank
    if config.is_moe and info.size > 1:
        from minisgl.layers.moe import expert_range

        first, count = expert_range(config.num_experts)
        if count < config.num_experts:
            ep = (first, count)
    n_local = ep[1] if ep else config.num_experts
    for path in files:
        with safetensors.safe_open(path, framework="pt", device=str(device)) as f:
            for name in f.keys():
                if name.startswith(("vision_tower.", "multi_modal_projector.", "model.visual.")):
                    continue
                raw = f.get_tensor(name)
                key = name.removeprefix("language_model.")
                em = _EXPERT.match(key) if ".experts." in key else None
                if ep is not None and em is not None:  # per-expert tensor under EP: keep ours, whole
                    e = int(em.group("idx"))
                    if not ep[0] <= e < ep[0] + ep[1]:
                        del raw
                        continue
                    key = f"{em.group('pre')}.{e - ep[0]}.{em.group('name')}"
                if ".experts." in key and em is None:
                    conv = _fused_expert(key, raw, pending, info.rank, info.size, dtype, ep)
                    if conv is None:
                        continue
                    if isinstance(conv, list):
                        yield from conv
                        continue
                    if conv is not False:
                        yield conv
                        continue
                if ep is not None and em is not None:
                    t = raw
                else:
                    t = shard_tensor(key, raw, info.rank, info.size, config.num_kv_heads, config.head_dim)
                    if key.endswith(".down_proj.weight") and ".experts." not in key:
                        t = _pad_to_block(t, t.dim() - 1)  # dense MLP: match the padded gate/up rows
                del raw
                mi = _merge_slot(key)
                if mi is not None:
                    mkey, slot, slots = mi
                    merge.setdefault(mkey, {})[slot] = t
                    if any(s not in merge[mkey] for s in slots):
                        continue
                    key, t = mkey, _finish_merge(mkey, merge.pop(mkey))
                ei = _expert_key(key) if config.is_moe else None
                if ei is not None:
                    pkey, idx = ei
                    bucket = experts.setdefault(pkey, {})
                    bucket[idx] = t
                    if len(bucket) < n_local:
                        continue
                    del experts[pkey]
                    yield pkey, torch.stack([bucket[i] for i in range(n_local)])
                else:
                    yield key, t
    if merge or experts or pending:
        raise RuntimeError(f"incomplete checkpoint groups: {list(merge) + list(experts) + list(pending)}")
