"""Scheduler I/O (reference: python/minisgl/scheduler/io.py:15-133).

* single rank: PULL from the tokenizer, PUSH replies to the detokenizer;
* TP rank 0: PULL raw bytes, PUB them to the other ranks, and broadcast the message count over the
  gloo group every loop so all ranks take identical scheduling decisions;
* TP rank > 0: read the count, then SUB that many messages;
* offline: the subclass supplies ``offline_receive_msg`` / ``offline_send_result``.
"""

from __future__ import annotations

from typing import List

import torch

from minisgl.message import BaseBackendMsg, BaseTokenizerMsg, BatchTokenizerMsg, DetokenizeMsg
from minisgl.utils import init_logger

logger = init_logger(__name__)


class SchedulerIOMixin:
    def __init__(self, config, tp_cpu_group) -> None:
        from minisgl.utils.mp import ZmqPubQueue, ZmqPullQueue, ZmqPushQueue, ZmqSubQueue

        self.tp_cpu_group = tp_cpu_group
        info = config.tp_info
        self._queues = []
        if config.offline_mode:
            self.receive_msg = self.offline_receive_msg
            self.send_result = self.offline_send_result
            return
        if info.is_primary():
            self._recv_from_tokenizer = ZmqPullQueue(
                config.zmq_backend_addr, create=True, decoder=BaseBackendMsg.decoder
            )
            self._send_into_tokenizer = ZmqPushQueue(
                config.zmq_detokenizer_addr,
                create=config.scheduler_binds_detokenizer,
                encoder=BaseTokenizerMsg.encoder,
            )
            self._queues += [self._recv_from_tokenizer, self._send_into_tokenizer]
        recv, send = self._recv_single, self._reply_rank0
        if info.size > 1:
            if info.is_primary():
                self._send_into_ranks = ZmqPubQueue(
                    config.zmq_scheduler_broadcast_addr, create=True, encoder=BaseBackendMsg.encoder
                )
                self._queues.append(self._send_into_ranks)
                recv = self._recv_multi_rank0
            else:
                self._recv_from_rank0 = ZmqSubQueue(
                    config.zmq_scheduler_broadcast_addr, create=False, decoder=BaseBackendMsg.decoder
                )
                self._queues.append(self._recv_from_rank0)
                recv, send = self._recv_multi_rankn, self._reply_noop
        self.receive_msg = recv
        self.send_result = send

    # subclass hooks ---------------------------------------------------------
    def run_when_idle(self) -> None:
        pass

    def offline_receive_msg(self, blocking: bool = False) -> List[BaseBackendMsg]:
        raise NotImplementedError

    def offline_send_result(self, reply: List[DetokenizeMsg]) -> None:
        raise NotImplementedError

    def sync_all_ranks(self) -> None:
        if self.tp_cpu_group is not None:
            torch.distributed.barrier(group=self.tp_cpu_group)

    def stop_io(self) -> None:
        for q in self._queues:
            q.stop()
        self._queues = []

    # strategies -------------------------------------------------------------
    def _recv_single(self, blocking: bool = False) -> List[BaseBackendMsg]:
        out: List[BaseBackendMsg] = []
        if blocking:
            self.run_when_idle()
            out.append(self._recv_from_tokenizer.get())
        while not self._recv_from_tokenizer.empty():
            out.append(self._recv_from_tokenizer.get())
        return out

    def _recv_multi_rank0(self, blocking: bool = False) -> List[BaseBackendMsg]:
        out: List[BaseBackendMsg] = []
        if blocking:  # the first message is forwarded at once; peers block on SUB for it
            self.run_when_idle()
            raw = self._recv_from_tokenizer.get_raw()
            self._send_into_ranks.put_raw(raw)
            out.append(self._recv_from_tokenizer.decode(raw))
        raws: List[bytes] = []
        while not self._recv_from_tokenizer.empty():
            raws.append(self._recv_from_tokenizer.get_raw())
        count = torch.tensor([len(raws)], dtype=torch.int64)
        torch.distributed.broadcast(count, src=0, group=self.tp_cpu_group)
        for raw in raws:
            self._send_into_ranks.put_raw(raw)
            out.append(self._recv_from_tokenizer.decode(raw))
        return out

    def _recv_multi_rankn(self, blocking: bool = False) -> List[BaseBackendMsg]:
        out: List[BaseBackendMsg] = []
        if blocking:
            self.run_when_idle()
            out.append(self._recv_from_rank0.get())
        count = torch.tensor([-1], dtype=torch.int64)
        torch.distributed.broadcast(count, src=0, group=self.tp_cpu_group)
        out += [self._recv_from_rank0.get() for _ in range(int(count.item()))]
        return out

    def _reply_rank0(self, reply: List[DetokenizeMsg]) -> None:
        if len(reply) == 1:
            self._send_into_tokenizer.put(reply[0])
        elif reply:
            self._send_into_tokenizer.put(BatchTokenizerMsg(data=list(reply)))

    def _reply_noop(self, reply: List[DetokenizeMsg]) -> None:
        pass
