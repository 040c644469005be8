"""Streaming safetensors loader with tensor-parallel sharding
(reference: python/minisgl/models/weight.py:16-124).

Per tensor: strip the ``language_model.`` prefix, skip vision weights, take this rank's shard
(q/k/v/gate/up and their biases split on dim 0 with KV-head replication when tp > kv heads;
o/down split on dim 1; embed/lm_head split into ``ceil(V/tp)`` vocab rows, zero padded; sinks
split by head), merge q,k,v -> ``qkv_proj`` and gate,up -> ``gate_up_proj`` (gate/up interleaved
in 128-row blocks for the fused activation epilogue; expert weights keep plain ``[gate; up]``
halves), and stack per-expert tensors into packed
``[E, ...]`` tensors. Yields ``(name, tensor)`` already on the target device.
"""

from __future__ import annotations

import glob
import os
import re
from typing import Dict, Iterator, Tuple

import torch

from minisgl.ops.reference import interleave_gate_up
from minisgl.parallel import get_tp_info
from minisgl.utils import div_ceil

_DIM0 = (".q_proj.", ".k_proj.", ".v_proj.", ".gate_proj.", ".up_proj.")
_DIM1 = (".o_proj.weight", ".down_proj.weight")
_QKV = {".q_proj.": "q", ".k_proj.": "k", ".v_proj.": "v"}
_GU = {".gate_proj.": "gate", ".up_proj.": "up"}
_EXPERT = re.compile(r"^(?P<pre>.+\.experts)\.(?P<idx>\d+)\.(?P<name>.+)$")


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
    if "experts" in key and key.endswith("down_proj") and t.dim() == 3:
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


def _finish_merge(key: str, parts: Dict[str, torch.Tensor]) -> torch.Tensor:
    if "gate_up_proj" in key and ".experts." in key:  # experts keep [gate; up] halves
        return torch.cat([parts["gate"], parts["up"]], dim=0)
    if "gate_up_proj" in key:
        g, u = parts["gate"], parts["up"]
        if g.dim() == 1:  # bias
            return interleave_gate_up(g[:, None], u[:, None])[:, 0]
        return interleave_gate_up(g, u)
    return torch.cat([parts["q"], parts["k"], parts["v"]], dim=0)


def _expert_key(key: str):
    m = _EXPERT.match(key)
    if m is None:
        return None
    name = m.group("name").removesuffix(".weight")
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
    for path in files:
        with safetensors.safe_open(path, framework="pt", device=str(device)) as f:
            for name in f.keys():
                if name.startswith(("vision_tower.", "multi_modal_projector.", "model.visual.")):
                    continue
                raw = f.get_tensor(name)
                key = name.removeprefix("language_model.")
                t = shard_tensor(key, raw, info.rank, info.size, config.num_kv_heads, config.head_dim)
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
                    if len(bucket) < config.num_experts:
                        continue
                    del experts[pkey]
                    yield pkey, torch.stack([bucket[i] for i in range(config.num_experts)])
                else:
                    yield key, t
    if merge or experts:
        raise RuntimeError(f"incomplete checkpoint groups: {list(merge) + list(experts)}")
