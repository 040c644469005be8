"""Minimal module system (not ``nn.Module``): tensors held as public attributes form the state
dict, sub-ops nest by attribute name, ``_private`` attributes are skipped
(reference: python/minisgl/layers/base.py:15-99). Checkpoint key names therefore follow the
attribute paths, e.g. ``model.layers.3.self_attn.qkv_proj.weight``."""

from __future__ import annotations

from typing import Any, Dict, Generic, Iterator, List, Tuple, TypeVar

import torch

StateDict = Dict[str, torch.Tensor]


def _join(prefix: str, name: str) -> str:
    return f"{prefix}.{name}" if prefix else name


class BaseOP:
    def forward(self, *args: Any, **kwargs: Any) -> Any:
        raise NotImplementedError

    def named_children(self) -> Iterator[Tuple[str, Any]]:
        for name, v in vars(self).items():
            if not name.startswith("_"):
                yield name, v

    def state_dict(self, *, prefix: str = "", result: StateDict | None = None) -> StateDict:
        out = {} if result is None else result
        for name, v in self.named_children():
            if isinstance(v, torch.Tensor):
                out[_join(prefix, name)] = v
            elif isinstance(v, BaseOP):
                v.state_dict(prefix=_join(prefix, name), result=out)
        return out

    def load_state_dict(self, state_dict: StateDict, *, prefix: str = "", _internal: bool = False) -> None:
        for name, v in list(self.named_children()):
            key = _join(prefix, name)
            if isinstance(v, torch.Tensor):
                if key not in state_dict:
                    raise KeyError(f"missing weight {key}")
                item = state_dict.pop(key)
                if tuple(item.shape) != tuple(v.shape) or item.dtype != v.dtype:
                    raise ValueError(
                        f"{key}: expected {tuple(v.shape)} {v.dtype}, got {tuple(item.shape)} {item.dtype}"
                    )
                setattr(self, name, item)
            elif isinstance(v, BaseOP):
                v.load_state_dict(state_dict, prefix=key, _internal=True)
        if not _internal and state_dict:
            raise RuntimeError(f"unexpected weights: {sorted(state_dict)[:8]}")


class StateLessOP(BaseOP):
    def state_dict(self, *, prefix: str = "", result: StateDict | None = None) -> StateDict:
        return {} if result is None else result

    def load_state_dict(self, state_dict: StateDict, *, prefix: str = "", _internal: bool = False) -> None:
        if not _internal and state_dict:
            raise RuntimeError(f"unexpected weights: {sorted(state_dict)[:8]}")


T = TypeVar("T", bound=BaseOP)


class OPList(BaseOP, Generic[T]):
    def __init__(self, ops: List[T]):
        self.op_list = ops

    def state_dict(self, *, prefix: str = "", result: StateDict | None = None) -> StateDict:
        out = {} if result is None else result
        for i, op in enumerate(self.op_list):
            op.state_dict(prefix=_join(prefix, str(i)), result=out)
        return out

    def load_state_dict(self, state_dict: StateDict, *, prefix: str = "", _internal: bool = False) -> None:
        for i, op in enumerate(self.op_list):
            op.load_state_dict(state_dict, prefix=_join(prefix, str(i)), _internal=True)
        if not _internal and state_dict:
            raise RuntimeError(f"unexpected weights: {sorted(state_dict)[:8]}")

    def __iter__(self):
        return iter(self.op_list)

    def __len__(self) -> int:
        return len(self.op_list)
