import msgpack
import torch

from minisgl.core import SamplingParams
from minisgl.message import (
    AbortBackendMsg,
    BaseBackendMsg,
    BaseFrontendMsg,
    BaseTokenizerMsg,
    BatchBackendMsg,
    BatchTokenizerMsg,
    DetokenizeMsg,
    ExitMsg,
    TokenizeMsg,
    UserMsg,
    UserReply,
)


def roundtrip(msg, cls):
    raw = msgpack.packb(cls.encoder(msg), use_bin_type=True)
    return cls.decoder(msgpack.unpackb(raw, raw=False))


def test_backend_roundtrip():
    ids = torch.tensor([1, 2, 3, 40000], dtype=torch.int32)
    m = BatchBackendMsg(data=[
        UserMsg(uid=7, input_ids=ids, sampling_params=SamplingParams(temperature=0.5, top_k=3)),
        AbortBackendMsg(uid=3),
        ExitMsg(),
    ])
    out = roundtrip(m, BaseBackendMsg)
    assert isinstance(out, BatchBackendMsg) and len(out.data) == 3
    u = out.data[0]
    assert isinstance(u, UserMsg) and u.uid == 7
    assert u.input_ids.dtype == torch.int32 and torch.equal(u.input_ids, ids)
    assert u.sampling_params == SamplingParams(temperature=0.5, top_k=3)
    assert isinstance(out.data[1], AbortBackendMsg) and out.data[1].uid == 3
    assert isinstance(out.data[2], ExitMsg)


def test_tokenizer_frontend_roundtrip():
    m = BatchTokenizerMsg(data=[
        DetokenizeMsg(uid=1, next_token=5, finished=False),
        TokenizeMsg(uid=2, text=[{"role": "user", "content": "hi"}], sampling_params=SamplingParams()),
    ])
    out = roundtrip(m, BaseTokenizerMsg)
    assert out.data[0] == m.data[0] and out.data[1] == m.data[1]
    r = roundtrip(UserReply(uid=3, incremental_output="abc", finished=True), BaseFrontendMsg)
    assert r == UserReply(uid=3, incremental_output="abc", finished=True)
