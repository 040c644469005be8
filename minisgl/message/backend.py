"""Messages into the scheduler (reference: python/minisgl/message/backend.py:12-41)."""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List

import torch

from minisgl.core import SamplingParams

from .utils import deserialize_type, serialize_type


@dataclass
class BaseBackendMsg:
    def encoder(self) -> Dict:
        return serialize_type(self)

    @staticmethod
    def decoder(data: Dict) -> "BaseBackendMsg":
        return deserialize_type(_TABLE, data)


@dataclass
class BatchBackendMsg(BaseBackendMsg):
    data: List[BaseBackendMsg]


@dataclass
class ExitMsg(BaseBackendMsg):
    pass


@dataclass
class UserMsg(BaseBackendMsg):
    uid: int
    input_ids: torch.Tensor  # CPU 1-D int32
    sampling_params: SamplingParams


@dataclass
class AbortBackendMsg(BaseBackendMsg):
    uid: int


_TABLE = {
    c.__name__: c
    for c in (BatchBackendMsg, ExitMsg, UserMsg, AbortBackendMsg, SamplingParams)
}
