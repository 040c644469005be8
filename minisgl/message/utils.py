"""Reflective (de)serialization of message dataclasses to msgpack-able dicts.

Nested dataclasses carry a ``"__t"`` type tag resolved through a class table; 1-D CPU tensors are
sent as raw bytes plus dtype. Wire format is this engine's own; the behaviour matches the
reference (python/minisgl/message/utils.py:20-69).
"""

from __future__ import annotations

import dataclasses
from typing import Any, Dict, Type

import numpy as np
import torch

_TYPE_KEY = "__t"
_TENSOR = "tensor"
_NP_OF = {
    torch.int32: "int32",
    torch.int64: "int64",
    torch.float32: "float32",
    torch.float16: "float16",
    torch.uint8: "uint8",
    torch.bool: "bool",
}


def serialize_type(obj: Any) -> Any:
    if isinstance(obj, torch.Tensor):
        if obj.dim() != 1:
            raise ValueError("only 1-D tensors can be serialized")
        t = obj.detach().cpu().contiguous()
        return {_TYPE_KEY: _TENSOR, "dtype": _NP_OF[t.dtype], "data": t.numpy().tobytes()}
    if dataclasses.is_dataclass(obj) and not isinstance(obj, type):
        out: Dict[str, Any] = {_TYPE_KEY: type(obj).__name__}
        for f in dataclasses.fields(obj):
            if f.init:
                out[f.name] = serialize_type(getattr(obj, f.name))
        return out
    if isinstance(obj, dict):
        return {k: serialize_type(v) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return [serialize_type(v) for v in obj]
    if obj is None or isinstance(obj, (bool, int, float, str, bytes)):
        return obj
    raise TypeError(f"cannot serialize {type(obj).__name__}")


def deserialize_type(table: Dict[str, Type], data: Any) -> Any:
    if isinstance(data, dict):
        tag = data.get(_TYPE_KEY)
        if tag == _TENSOR:
            arr = np.frombuffer(data["data"], dtype=np.dtype(data["dtype"])).copy()
            return torch.from_numpy(arr)
        if tag is not None:
            cls = table.get(tag)
            if cls is None:
                raise KeyError(f"unknown message type {tag}")
            kwargs = {k: deserialize_type(table, v) for k, v in data.items() if k != _TYPE_KEY}
            return cls(**kwargs)
        return {k: deserialize_type(table, v) for k, v in data.items()}
    if isinstance(data, (list, tuple)):
        return [deserialize_type(table, v) for v in data]
    return data
