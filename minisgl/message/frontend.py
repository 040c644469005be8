"""Messages into the API server (reference: python/minisgl/message/frontend.py:9-29)."""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List

from .utils import deserialize_type, serialize_type


@dataclass
class BaseFrontendMsg:
    @staticmethod
    def encoder(msg: "BaseFrontendMsg") -> Dict:
        return serialize_type(msg)

    @staticmethod
    def decoder(data: Dict) -> "BaseFrontendMsg":
        return deserialize_type(_TABLE, data)


@dataclass
class BatchFrontendMsg(BaseFrontendMsg):
    data: List[BaseFrontendMsg]


@dataclass
class UserReply(BaseFrontendMsg):
    uid: int
    incremental_output: str
    finished: bool
    num_output_tokens: int = 0
    num_input_tokens: int = 0
    finish_reason: str = ""  # on the final reply: "stop" (EOS) or "length" (max_tokens / context)


_TABLE = {c.__name__: c for c in (BatchFrontendMsg, UserReply)}
