"""Messages into the tokenizer / detokenizer workers
(reference: python/minisgl/message/tokenizer.py:11-43)."""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List

from minisgl.core import SamplingParams

from .utils import deserialize_type, serialize_type


@dataclass
class BaseTokenizerMsg:
    @staticmethod
    def encoder(msg: "BaseTokenizerMsg") -> Dict:
        return serialize_type(msg)

    @staticmethod
    def decoder(data: Dict) -> "BaseTokenizerMsg":
        return deserialize_type(_TABLE, data)


@dataclass
class BatchTokenizerMsg(BaseTokenizerMsg):
    data: List[BaseTokenizerMsg]


@dataclass
class DetokenizeMsg(BaseTokenizerMsg):
    uid: int
    next_token: int
    finished: bool
    eos: bool = False  # the request stopped on this EOS token (not part of the output)


@dataclass
class TokenizeMsg(BaseTokenizerMsg):
    uid: int
    text: str | List[Dict[str, str]]
    sampling_params: SamplingParams


@dataclass
class AbortMsg(BaseTokenizerMsg):
    uid: int


_TABLE = {
    c.__name__: c
    for c in (BatchTokenizerMsg, DetokenizeMsg, TokenizeMsg, AbortMsg, SamplingParams)
}
