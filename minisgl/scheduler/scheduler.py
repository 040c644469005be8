"""Per-rank scheduler loop (reference: python/minisgl/scheduler/scheduler.py:45-267).

Overlap mode (default): while the engine stream computes batch N, the host receives messages,
schedules and uploads batch N+1 on the scheduler stream, launches it, and only then processes
N's sampled tokens. Invariants kept from the reference design:

* sampled tokens stay on the device (``engine.last_tokens``) and feed the next decode directly;
* ``Req.complete_one`` advances lengths at launch, so N+1 is planned as if N's token existed;
* a finished request may run one extra decode step; ``finished_reqs`` prevents a double free;
* a ``ForwardInput`` keeps the host/device plan alive until its results are processed.
"""

from __future__ import annotations

from typing import List, NamedTuple, Set, Tuple

import torch

from minisgl.core import UNBOUNDED_MAX_TOKENS, Batch, Req
from minisgl.env import ENV
from minisgl.message import (
    AbortBackendMsg,
    BaseBackendMsg,
    BatchBackendMsg,
    DetokenizeMsg,
    ExitMsg,
    UserMsg,
)
from minisgl.utils import init_logger

from .cache import CacheManager
from .config import SchedulerConfig
from .decode import DecodeManager
from .io import SchedulerIOMixin
from .prefill import ChunkedReq, PrefillManager
from .table import TableManager

logger = init_logger(__name__)


class ForwardInput(NamedTuple):
    batch: Batch
    sample_args: object
    plan: object
    dev: dict


ForwardData = Tuple[ForwardInput, object]


class Scheduler(SchedulerIOMixin):
    def __init__(self, config: SchedulerConfig):
        from minisgl.engine import Engine

        self.config = config
        self.engine = Engine(config)
        self.device = self.engine.device
        if self.engine.is_cuda:
            self.stream = torch.cuda.Stream(device=self.device)
            torch.cuda.set_stream(self.stream)
        else:
            self.stream = None
        self.table_manager = TableManager(config.max_running_req, self.engine.page_table)
        self.cache_manager = CacheManager(self.engine.num_pages, config.page_size, config.cache_type)
        self.decode_manager = DecodeManager(config.page_size)
        self.prefill_manager = PrefillManager(self.cache_manager, self.table_manager, self.decode_manager)
        self.finished_reqs: Set[Req] = set()
        from minisgl.utils.hf import load_tokenizer

        self.tokenizer = load_tokenizer(config.model_path)
        self.eos_token_id = self.tokenizer.eos_token_id
        self.prefill_budget = config.max_extend_tokens
        super().__init__(config, self.engine.tp_cpu_group)

    # ------------------------------------------------------------------ loops
    def run_when_idle(self) -> None:
        logger.info_rank0("Scheduler idle, waiting for requests...")
        self.cache_manager.check_integrity()

    def overlap_loop(self, last: ForwardData | None) -> ForwardData | None:
        blocking = last is None and not (self.prefill_manager.runnable or self.decode_manager.runnable)
        for msg in self.receive_msg(blocking=blocking):
            self._process_one_msg(msg)
        fi = self._schedule_next_batch()
        ongoing = None
        if fi is not None:
            with self.engine.stream_ctx():
                if self.engine.is_cuda:
                    self.engine.stream.wait_stream(self.stream)
                ongoing = (fi, self._forward(fi))
        self._process_last_data(last)
        return ongoing

    def normal_loop(self) -> None:
        blocking = not (self.prefill_manager.runnable or self.decode_manager.runnable)
        for msg in self.receive_msg(blocking=blocking):
            self._process_one_msg(msg)
        fi = self._schedule_next_batch()
        if fi is not None:
            self._process_last_data((fi, self._forward(fi)))

    @torch.inference_mode()
    def run_forever(self):
        if ENV.DISABLE_OVERLAP_SCHEDULING or not self.engine.is_cuda:
            with self.engine.stream_ctx():
                while True:
                    self.normal_loop()
        else:
            torch.cuda.set_stream(self.stream)
            data = None
            while True:
                data = self.overlap_loop(data)

    def shutdown(self) -> None:
        if self.engine.is_cuda:
            torch.cuda.synchronize(self.device)
        self.sync_all_ranks()
        self.stop_io()
        self.engine.shutdown()

    # ------------------------------------------------------------------ results
    def _process_last_data(self, last: ForwardData | None) -> None:
        if last is None:
            return
        fi, out = last
        batch = fi.batch
        out.copy_done_event.synchronize()
        tokens = out.next_tokens_cpu.tolist()
        reply: List[DetokenizeMsg] = []
        newly_finished: Set[Req] = set()
        with self.cache_manager.lazy_free_region():
            eos = self.eos_token_id
            for req, tok in zip(batch.reqs, tokens):
                if isinstance(req, ChunkedReq) or req.aborted:
                    continue
                if req in self.finished_reqs:
                    # Stopped on EOS in the previous batch, after this batch was already launched
                    # (overlap scheduling): this token is surplus. The reference still sends it
                    # (python/minisgl/scheduler/scheduler.py:147-164), which adds a token after
                    # EOS to offline outputs.
                    continue
                req.append_host(tok)
                stop_eos = tok == eos and not req.sampling_params.ignore_eos
                finished = stop_eos or req.host_len >= req.max_device_len
                reply.append(DetokenizeMsg(uid=req.uid, next_token=tok, finished=finished, eos=stop_eos))
                if finished:
                    self.decode_manager.remove_req(req)
                    self._free_req_resources(req)
                    newly_finished.add(req)
                elif batch.is_prefill and not finished:
                    self.cache_manager.cache_req(req, finished=False)
        self.finished_reqs = newly_finished
        self.send_result(reply)
        if ENV.DEBUG_CHECK_INTEGRITY:
            self.cache_manager.prefix_cache.check_integrity()

    def _process_one_msg(self, msg: BaseBackendMsg) -> None:
        if isinstance(msg, BatchBackendMsg):
            for m in msg.data:
                self._process_one_msg(m)
        elif isinstance(msg, ExitMsg):
            raise KeyboardInterrupt
        elif isinstance(msg, UserMsg):
            n, cap = len(msg.input_ids), self.engine.max_seq_len
            reason = ("empty prompt" if n == 0 else f"input length {n} >= {cap}" if n >= cap else
                      "max_tokens < 1" if msg.sampling_params.max_tokens < 1 else None)
            if reason is not None:
                # finish it at once with no output, so that its client is answered
                logger.warning_rank0(f"request {msg.uid} rejected: {reason}")
                self.send_result([DetokenizeMsg(uid=msg.uid, next_token=0, finished=True, eos=True)])
                return
            if msg.sampling_params.max_tokens > cap - n:
                if msg.sampling_params.max_tokens < UNBOUNDED_MAX_TOKENS:
                    logger.warning_rank0(f"request {msg.uid}: max_tokens clamped to {cap - n}")
                msg.sampling_params.max_tokens = cap - n
            self.prefill_manager.add_one_req(msg)
        elif isinstance(msg, AbortBackendMsg):
            req = self.prefill_manager.abort_req(msg.uid) or self.decode_manager.abort_req(msg.uid)
            if req is not None:
                # a batch holding the request may still be in flight (overlap scheduling): its
                # result for this request is dropped, so the resources are released only here
                req.aborted = True
                self._free_req_resources(req)
        else:
            raise NotImplementedError(f"unknown message {type(msg).__name__}")

    def _free_req_resources(self, req: Req) -> None:
        self.table_manager.free(req.table_idx)
        self.cache_manager.cache_req(req, finished=True)

    # ------------------------------------------------------------------ scheduling
    def _schedule_next_batch(self) -> ForwardInput | None:
        batch = (
            self.prefill_manager.schedule_next_batch(self.prefill_budget)
            or self.decode_manager.schedule_next_batch()
        )
        return self._prepare_batch(batch) if batch is not None else None

    def _prepare_batch(self, batch: Batch) -> ForwardInput:
        from minisgl.engine import BatchPlan

        eng = self.engine
        eng.graph_runner.pad_batch(batch)
        pt = self.cache_manager.allocate_paged(batch.reqs)
        plan = BatchPlan(batch, pt, eng.junk_row)
        dev = eng.upload_plan(batch, plan)
        args = eng.sampler.prepare(batch)
        return ForwardInput(batch, args, plan, dev)

    def _forward(self, fi: ForwardInput):
        out = self.engine.forward_batch(fi.batch, fi.sample_args, fi.dev)
        self.decode_manager.filter_reqs(fi.batch.reqs)
        return out
