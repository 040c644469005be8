"""Tokenizer / detokenizer worker process (reference: python/minisgl/tokenizer/server.py:30-110).

Pulls batches of messages, and routes: TokenizeMsg -> UserMsg to the scheduler, DetokenizeMsg ->
UserReply to the API server, AbortMsg -> AbortBackendMsg to the scheduler.
"""

from __future__ import annotations

from typing import List

import torch

from minisgl.message import (
    AbortBackendMsg,
    AbortMsg,
    BaseBackendMsg,
    BaseFrontendMsg,
    BaseTokenizerMsg,
    BatchBackendMsg,
    BatchFrontendMsg,
    BatchTokenizerMsg,
    DetokenizeMsg,
    TokenizeMsg,
    UserMsg,
    UserReply,
)
from minisgl.utils import init_logger


def _flatten(msg) -> List[BaseTokenizerMsg]:
    return list(msg.data) if isinstance(msg, BatchTokenizerMsg) else [msg]


def _one_or_batch(items, batch_cls):
    return items[0] if len(items) == 1 else batch_cls(data=items)


@torch.inference_mode()
def tokenize_worker(*, tokenizer_path: str, addr: str, create: bool, backend_addr: str, frontend_addr: str,
                    local_bs: int, tokenizer_id: int = -1, model_source: str = "huggingface",
                    ack_queue=None) -> None:
    from minisgl.utils.hf import load_tokenizer
    from minisgl.utils.mp import ZmqPullQueue, ZmqPushQueue
    from minisgl.utils.proc import die_with_parent

    die_with_parent()  # the worker never outlives the server process that spawned it

    from .detokenize import DetokenizeManager
    from .tokenize import TokenizeManager

    logger = init_logger(__name__, f"tokenizer_{tokenizer_id}")
    to_backend = ZmqPushQueue(backend_addr, create=False, encoder=BaseBackendMsg.encoder)
    to_frontend = ZmqPushQueue(frontend_addr, create=False, encoder=BaseFrontendMsg.encoder)
    inbox = ZmqPullQueue(addr, create=create, decoder=BaseTokenizerMsg.decoder)
    tokenizer = load_tokenizer(tokenizer_path)
    tok, detok = TokenizeManager(tokenizer), DetokenizeManager(tokenizer)
    if ack_queue is not None:
        ack_queue.put(f"tokenizer {tokenizer_id} ready")
    try:
        while True:
            pending = _flatten(inbox.get())
            while len(pending) < local_bs and not inbox.empty():
                pending += _flatten(inbox.get())
            detoks = [m for m in pending if isinstance(m, DetokenizeMsg)]
            toks = [m for m in pending if isinstance(m, TokenizeMsg)]
            aborts = [m for m in pending if isinstance(m, AbortMsg)]
            if detoks:
                texts = detok.detokenize(detoks)
                to_frontend.put(_one_or_batch(
                    [UserReply(uid=m.uid, incremental_output=t, finished=m.finished,
                               finish_reason=("stop" if m.eos else "length") if m.finished else "")
                     for m, t in zip(detoks, texts)],
                    BatchFrontendMsg))
            if toks:
                ids = tok.tokenize(toks)
                to_backend.put(_one_or_batch(
                    [UserMsg(uid=m.uid, input_ids=t, sampling_params=m.sampling_params) for m, t in zip(toks, ids)],
                    BatchBackendMsg))
                # the prompt length, for the response's usage (a reply without text)
                to_frontend.put(_one_or_batch(
                    [UserReply(uid=m.uid, incremental_output="", finished=False, num_input_tokens=max(1, len(t)))
                     for m, t in zip(toks, ids)], BatchFrontendMsg))
            if aborts:
                to_backend.put(_one_or_batch([AbortBackendMsg(uid=m.uid) for m in aborts], BatchBackendMsg))
            logger.debug(f"handled {len(detoks)} detok / {len(toks)} tok / {len(aborts)} abort")
    except KeyboardInterrupt:
        pass
