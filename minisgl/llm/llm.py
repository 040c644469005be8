"""Offline API: ``LLM(model_path, **config).generate(prompts, sampling_params)``
(reference: python/minisgl/llm/llm.py:28-98).

Runs an in-process scheduler in offline mode. Under ``torchrun`` (``WORLD_SIZE > 1``) every rank
constructs the same ``LLM`` with the same prompts and the ranks form one tensor-parallel group.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Dict, List, Tuple

import torch

from minisgl.core import SamplingParams
from minisgl.message import BaseBackendMsg, DetokenizeMsg, UserMsg
from minisgl.parallel import DistributedInfo
from minisgl.scheduler import Scheduler, SchedulerConfig


class RequestAllFinished(Exception):
    pass


@dataclass
class RequestStatus:
    uid: int
    input_ids: List[int]
    output_ids: List[int]


def _tp_from_env() -> Tuple[DistributedInfo, bool]:
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    if ws > 1:
        return DistributedInfo(int(os.environ["RANK"]), ws), True
    return DistributedInfo(0, 1), False


class LLM(Scheduler):
    def __init__(self, model_path: str, dtype: torch.dtype = torch.bfloat16, **kwargs):
        info, external = _tp_from_env()
        kwargs.setdefault("tp_info", info)
        kwargs.setdefault("external_process_group", external)
        config = SchedulerConfig(model_path=model_path, dtype=dtype, offline_mode=True, **kwargs)
        super().__init__(config)
        self.pending_requests: List[Tuple[List[int] | str, SamplingParams]] = []
        self.status_map: Dict[int, RequestStatus] = {}
        self.counter = 0

    def _tokenize_one(self, prompt) -> torch.Tensor:
        if isinstance(prompt, str):
            return torch.tensor(self.tokenizer.encode(prompt), dtype=torch.int32)
        if isinstance(prompt, torch.Tensor):
            return prompt.to("cpu", torch.int32).reshape(-1)
        return torch.tensor(prompt, dtype=torch.int32)

    def offline_receive_msg(self, blocking: bool = False) -> List[BaseBackendMsg]:
        if blocking and not self.pending_requests:
            raise RequestAllFinished()
        out: List[BaseBackendMsg] = []
        total = 0
        taken = 0
        for prompt, sp in self.pending_requests:
            if total >= self.prefill_budget:
                break
            ids = self._tokenize_one(prompt)
            total += len(ids)
            uid = self.counter + taken
            taken += 1
            out.append(UserMsg(uid=uid, input_ids=ids, sampling_params=SamplingParams(**vars(sp))))
            self.status_map[uid] = RequestStatus(uid, ids.tolist(), [])
        self.counter += taken
        self.pending_requests = self.pending_requests[taken:]
        return out

    def offline_send_result(self, reply: List[DetokenizeMsg]) -> None:
        for msg in reply:
            st = self.status_map[msg.uid]
            if not msg.eos:  # a stopping EOS is not output; with ignore_eos it is an ordinary token
                st.output_ids.append(msg.next_token)

    def generate(self, prompts, sampling_params) -> List[Dict[str, object]]:
        self.pending_requests = []
        self.status_map = {}
        self.counter = 0
        if isinstance(sampling_params, SamplingParams):
            sampling_params = [sampling_params] * len(prompts)
        self.pending_requests = list(zip(prompts, sampling_params))
        try:
            self.run_forever()
        except RequestAllFinished:
            pass
        results = []
        for i in range(len(prompts)):
            st = self.status_map[i]
            results.append({"text": self.tokenizer.decode(st.output_ids), "token_ids": st.output_ids})
        return results
