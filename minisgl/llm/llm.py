"""Offline API: ``LLM(model_path, **config).generate(prompts, sampling_params)``
(reference: python/minisgl/llm/llm.py:28-98; the constructor and ``generate`` signatures and the
``[{"text", "token_ids"}]`` result are that file's public surface).

``LLM`` is a scheduler in offline mode: instead of a ZeroMQ socket its input is a queue of the
prompts handed to ``generate``, released in slices of about one prefill chunk's worth of prompt
tokens whenever the scheduler polls, and its output is a per-request token list. The scheduler loop
ends (``RequestAllFinished``) when it would block with nothing queued. Under ``torchrun``
(``WORLD_SIZE > 1``) every rank constructs the same ``LLM``, gets the same prompts and runs the same
schedule; the ranks form one tensor-parallel group.
"""

from __future__ import annotations

import collections
import dataclasses
import os
from typing import Deque, Dict, List, Sequence, Tuple

import torch

from minisgl.core import SamplingParams
from minisgl.message import BaseBackendMsg, DetokenizeMsg, UserMsg
from minisgl.parallel import DistributedInfo
from minisgl.scheduler import Scheduler, SchedulerConfig


class RequestAllFinished(Exception):
    """Raised by the offline input when the scheduler waits for work and none is queued."""


def _rank_from_env() -> Tuple[DistributedInfo, bool]:
    """(tp_info, launched by torchrun) from the launcher's environment."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world <= 1:
        return DistributedInfo(0, 1), False
    return DistributedInfo(int(os.environ["RANK"]), world), True


class LLM(Scheduler):
    def __init__(self, model_path: str, dtype: torch.dtype = torch.bfloat16, **kwargs):
        info, external = _rank_from_env()
        kwargs.setdefault("tp_info", info)
        kwargs.setdefault("external_process_group", external)
        super().__init__(SchedulerConfig(model_path=model_path, dtype=dtype, offline_mode=True, **kwargs))
        self._queue: Deque[Tuple[int, object, SamplingParams]] = collections.deque()
        self._outputs: Dict[int, List[int]] = {}

    def _as_ids(self, prompt) -> torch.Tensor:
        if isinstance(prompt, str):
            return torch.tensor(self.tokenizer.encode(prompt), dtype=torch.int32)
        if isinstance(prompt, torch.Tensor):
            return prompt.to("cpu", torch.int32).reshape(-1)
        return torch.tensor(prompt, dtype=torch.int32)

    def offline_receive_msg(self, blocking: bool = False) -> List[BaseBackendMsg]:
        if not self._queue:
            if blocking:
                raise RequestAllFinished()
            return []
        msgs: List[BaseBackendMsg] = []
        tokens = 0
        while self._queue and tokens < self.prefill_budget:
            uid, prompt, sp = self._queue.popleft()
            ids = self._as_ids(prompt)
            tokens += int(ids.numel())
            # the scheduler may clamp max_tokens; the caller's object stays untouched
            msgs.append(UserMsg(uid=uid, input_ids=ids, sampling_params=dataclasses.replace(sp)))
        return msgs

    def offline_send_result(self, reply: List[DetokenizeMsg]) -> None:
        for msg in reply:
            if not msg.eos:  # a stopping EOS is not output; with ignore_eos it is an ordinary token
                self._outputs[msg.uid].append(msg.next_token)

    def generate(self, prompts: Sequence, sampling_params: SamplingParams | Sequence[SamplingParams]
                 ) -> List[Dict[str, object]]:
        if isinstance(sampling_params, SamplingParams):
            sampling_params = [sampling_params] * len(prompts)
        if len(sampling_params) != len(prompts):
            raise ValueError(f"{len(prompts)} prompts but {len(sampling_params)} sampling params")
        self._queue = collections.deque((uid, p, sp) for uid, (p, sp) in enumerate(zip(prompts, sampling_params)))
        self._outputs = {uid: [] for uid in range(len(prompts))}
        try:
            self.run_forever()
        except RequestAllFinished:
            pass
        return [{"text": self.tokenizer.decode(ids), "token_ids": ids}
                for ids in (self._outputs[uid] for uid in range(len(prompts)))]
