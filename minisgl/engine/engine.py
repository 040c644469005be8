"""Per-rank runtime: model + paged KV pool + attention/MoE backends + sampler + decode graphs
(reference: python/minisgl/engine/engine.py:29-233).

Batch metadata reaches the device as ONE packed int32 upload (``BatchPlan``, built on the host by
the scheduler); one kernel then applies its page-table writes and gathers ``out_loc``
(``csrc/kernels/plan.cu``).
Decode input ids come from ``last_tokens`` (one int32 per page-table row, written by the sampler),
so a decode step never waits for the host.
"""

from __future__ import annotations

import contextlib
import os
from datetime import timedelta
from typing import Dict, NamedTuple, Tuple

import numpy as np
import torch
import torch.distributed as dist

from minisgl._native import cuda as _cuda
from minisgl.attention import create_attention_backend
from minisgl.attention.paged import PAGED_DECODE_PAGES
from minisgl.core import Batch, Context, Req, SamplingParams, reset_global_ctx, set_global_ctx
from minisgl.env import ENV
from minisgl.kvcache import create_kvcache_pool
from minisgl.layers import set_rope_device
from minisgl.models import create_model, load_weight
from minisgl.parallel import destroy_distributed, set_torch_group, set_tp_info
from minisgl.parallel.info import reset_tp_info
from minisgl.utils import div_even, init_logger, torch_dtype

from .config import EngineConfig
from .counters import COUNTERS
from .graph import GraphRunner, determine_graph_bs
from .sample import BatchSamplingArgs, Sampler

logger = init_logger(__name__)


class ForwardOutput(NamedTuple):
    next_tokens_gpu: torch.Tensor
    next_tokens_cpu: torch.Tensor
    copy_done_event: object


class _HostEvent:
    def synchronize(self) -> None:
        pass


def _align32(n: int) -> int:
    return (n + 31) // 32 * 32


class Engine:
    def __init__(self, config: EngineConfig):
        self.config = config
        self.counters = COUNTERS
        info = config.tp_info
        set_tp_info(info.rank, info.size)
        self.device = torch.device(config.device or f"cuda:{info.rank}")
        self.is_cuda = self.device.type == "cuda"
        if self.is_cuda and config.page_size not in PAGED_DECODE_PAGES:
            # The decode kernel streams whole pages with TMA, so CUDA runs use 16/32/64-token pages
            # (the reference applies the same rule to its B200 backend:
            # python/minisgl/engine/engine.py, _adjust_config).
            logger.warning_rank0(f"page size {config.page_size} overridden to 64 (CUDA decode needs 16, 32 or 64)")
            object.__setattr__(config, "page_size", 64)
        if self.is_cuda and config.dtype == torch.float16:
            # the sm_100a kernels are written for bf16 activations and weights (same width, wider
            # range); float16 requests, including "auto" on float16/float32 checkpoints, run in bf16
            logger.warning_rank0("dtype float16 served as bfloat16 on CUDA")
            object.__setattr__(config, "dtype", torch.bfloat16)
        torch.manual_seed(config.seed)
        if self.is_cuda:
            torch.cuda.set_device(self.device)
            self.stream = torch.cuda.Stream(device=self.device)
            torch.cuda.set_stream(self.stream)
        else:
            self.stream = None
        self.dtype = config.dtype
        self.model_config = config.model_config
        self.ctx = Context(config.page_size)
        reset_global_ctx(None)
        set_global_ctx(self.ctx)

        self.tp_cpu_group = self._init_communication(config)
        free0 = self._sync_free_memory()[1]

        # ----------------------------------------------------------------- model
        set_rope_device(self.device)
        with torch.device("meta"), torch_dtype(config.dtype):
            self.model = create_model(self.model_config)
        self.model.load_state_dict(self._weights(config))

        # ----------------------------------------------------------------- KV pool
        self.num_pages = self._num_pages(free0)
        ps = config.page_size
        self.ctx.kv_cache = self.kv_cache = create_kvcache_pool(
            self.model_config, self.num_pages + 1, ps, self.dtype, self.device
        )
        self.dummy_slot = self.num_pages * ps
        num_tokens = self.num_pages * ps
        self.max_seq_len = min(config.max_seq_len, num_tokens)
        self.aligned_max_seq_len = _align32(self.max_seq_len)
        rows = config.max_running_req + 1  # + dummy row for graph padding
        self.dummy_row = config.max_running_req
        self.junk_row = config.max_running_req + 1  # sink for tokens that are never read
        self.ctx.page_table = self.page_table = torch.full(
            (rows, self.aligned_max_seq_len), self.dummy_slot, dtype=torch.int32, device=self.device
        )
        self.last_tokens = torch.zeros(rows + 1, dtype=torch.int32, device=self.device)

        # ----------------------------------------------------------------- backends
        self.ctx.attn_backend = self.attn_backend = create_attention_backend(
            config.attention_backend, self.model_config, self.device
        )
        if self.model_config.is_moe:
            from minisgl.moe import create_moe_backend

            self.ctx.moe_backend = self.moe_backend = create_moe_backend(config.moe_backend)
        self.sampler = Sampler(self.device, self.model_config.vocab_size)
        self._init_peer_comm(config)
        self._lm_shard = None
        lm_head = getattr(self.model, "lm_head", None)
        if config.tp_info.size > 1 and hasattr(lm_head, "return_local"):
            from minisgl.parallel import DistributedCommunicator

            lm_head.return_local = True
            self._lm_shard = (lm_head.vocab_shard, config.tp_info.size, DistributedCommunicator())

        # The decode graphs end at the final norm and the LM head runs after them, so a greedy batch
        # can take its argmax inside the LM-head GEMM (no logits written) and a sampled one gets logits.
        self._split_lm_head = self.is_cuda and hasattr(self.model, "forward_hidden")
        self._fused_greedy = self._split_lm_head and bool(ENV.FUSED_LM_HEAD)

        # ----------------------------------------------------------------- graphs
        self.dummy_req = Req(
            input_ids=torch.zeros(1, dtype=torch.int32), table_idx=self.dummy_row, cached_len=0,
            output_len=1, uid=-1, sampling_params=SamplingParams(), cache_handle=None,  # type: ignore[arg-type]
        )
        self.dummy_req.slots = np.array([self.dummy_slot], dtype=np.int32)
        graph_bs = determine_graph_bs(config.cuda_graph_bs, config.cuda_graph_max_bs, free0,
                                      config.max_running_req) if self.is_cuda else []
        self.graph_runner = GraphRunner(self, graph_bs, self.dummy_req)
        logger.info_rank0(
            f"Engine ready: {num_tokens} KV tokens, max_seq_len {self.max_seq_len}, device {self.device}"
        )

    # ===================================================================== setup helpers
    def _init_communication(self, config: EngineConfig):
        info = config.tp_info
        timeout = timedelta(seconds=config.distributed_timeout)
        if config.external_process_group or dist.is_initialized():
            # launched under torchrun: the default group exists (NCCL on GPU, gloo on CPU)
            if not dist.is_initialized():
                dist.init_process_group(backend="nccl" if self.is_cuda else "gloo", timeout=timeout)
            world = dist.group.WORLD
            cpu_group = dist.new_group(backend="gloo", timeout=timeout) if self.is_cuda else world
            set_torch_group(world)
            return cpu_group
        backend = "nccl" if (self.is_cuda and info.size > 1) else "gloo"
        if self.is_cuda and info.size > 1:
            os.environ.setdefault("NCCL_CUMEM_ENABLE", "1")
        dist.init_process_group(backend=backend, rank=info.rank, world_size=info.size,
                                timeout=timeout, init_method=config.distributed_addr)
        world = dist.group.WORLD
        cpu_group = dist.new_group(backend="gloo", timeout=timeout) if backend == "nccl" else world
        set_torch_group(world)
        return cpu_group

    def _init_peer_comm(self, config: EngineConfig) -> None:
        if not self.is_cuda or config.tp_info.size == 1:
            return
        mode = config.comm if config.comm != "auto" else ENV.COMM_MODE
        if mode == "nccl":
            return
        if mode in ("auto", "peer", "fused"):
            from minisgl.parallel.peer import enable_peer_comm

            # all-reduce messages are [tokens, hidden]; the LM-head gather is [bs, vocab/tp] fp32
            max_bytes = max(config.max_forward_len * self.model_config.hidden_size * self.dtype.itemsize,
                            config.max_running_req * self.model_config.vocab_size * 4 // config.tp_info.size)
            max_bytes = min(max_bytes, int(ENV.PYNCCL_MAX_BUFFER_SIZE))
            enable_peer_comm(self.tp_cpu_group, self.device, max_bytes, strict=(mode == "peer"))
        if mode in ("auto", "fused"):
            from minisgl.parallel.nvls import enable_nvls_norm

            # decode-sized activations (and short prefill chunks): [tokens, hidden] bf16
            rows = max(config.max_running_req, 1024)
            enable_nvls_norm(dist.group.WORLD, self.tp_cpu_group, self.device,
                             rows * self.model_config.hidden_size * self.dtype.itemsize, strict=(mode == "fused"))

    def _weights(self, config: EngineConfig) -> Dict[str, torch.Tensor]:
        if config.use_dummy_weight:
            g = torch.Generator(device=self.device).manual_seed(config.seed + config.tp_info.rank)
            out = {}
            fp4 = self._dummy_mxfp4()
            for k, v in self.model.state_dict().items():
                if fp4 and k.endswith((".experts.gate_up_proj", ".experts.down_proj")) and v.shape[2] % 64 == 0:
                    # MXFP4 checkpoint kept in fp4: random e2m1 bytes, scales near 2^-6 (|w| ~ 0.02)
                    blocks = torch.empty(*v.shape[:2], v.shape[2] // 32, 16, dtype=torch.uint8, device=self.device)
                    out[k + "_blocks"] = blocks.random_(0, 256, generator=g)
                    scales = torch.empty(*v.shape[:2], v.shape[2] // 32, dtype=torch.uint8, device=self.device)
                    out[k + "_scales"] = scales.random_(119, 123, generator=g)
                    continue
                if k.endswith(("norm.weight",)):
                    out[k] = torch.ones(v.shape, dtype=v.dtype, device=self.device)
                else:
                    t = torch.empty(v.shape, dtype=v.dtype, device=self.device)
                    if t.is_floating_point():
                        t.normal_(0.0, config.dummy_weight_std, generator=g)
                    else:
                        t.random_(0, 256, generator=g)
                    out[k] = t
            return out
        return {k: v.to(self.dtype) if v.is_floating_point() and not k.endswith("sinks") else v
                for k, v in load_weight(config.model_path, self.device, self.model_config)}

    def _dummy_mxfp4(self) -> bool:
        """Dummy weights for an MXFP4 checkpoint's experts are generated in fp4 (kept that way on
        the GPU) instead of bf16."""
        from minisgl.env import ENV

        return self.is_cuda and bool(ENV.MXFP4_RESIDENT) and getattr(self.model_config, "quant_method", None) == "mxfp4"

    def _sync_free_memory(self) -> Tuple[int, int]:
        if not self.is_cuda:
            return (1 << 40, 1 << 40)
        torch.cuda.synchronize(self.device)
        torch.cuda.empty_cache()
        free = torch.cuda.mem_get_info(self.device)[0]
        t = torch.tensor([free, -free], dtype=torch.int64)
        dist.all_reduce(t, op=dist.ReduceOp.MIN, group=self.tp_cpu_group)
        lo, hi = int(t[0]), -int(t[1])
        if hi - lo > 2 * (1 << 30):
            raise RuntimeError(f"free memory differs across TP ranks: min {lo}, max {hi}")
        return lo, hi

    def _num_pages(self, free_before: int) -> int:
        cfg = self.config
        mc = self.model_config
        kvh = div_even(mc.num_kv_heads, cfg.tp_info.size, allow_replicate=True)
        per_page = 2 * mc.head_dim * kvh * cfg.page_size * self.dtype.itemsize * mc.num_layers
        if cfg.num_page_override is not None:
            n = cfg.num_page_override
        elif not self.is_cuda:
            n = max(8192 // cfg.page_size, 2)
        else:
            free_after = self._sync_free_memory()[1]
            model_bytes = free_before - free_after
            n = int(cfg.memory_ratio * free_before - model_bytes) // per_page
        if n <= 1:
            raise RuntimeError("not enough memory for the KV cache; lower --memory-ratio or --num-pages")
        logger.info_rank0(f"KV cache: {n * cfg.page_size} tokens, {n * per_page / (1 << 30):.2f} GiB")
        return n

    # ===================================================================== per batch
    def stream_ctx(self):
        return torch.cuda.stream(self.stream) if self.is_cuda else contextlib.nullcontext()

    def upload_plan(self, batch: Batch, plan: "BatchPlan") -> dict:
        """Copy the packed plan to the device, apply page-table writes, derive out_loc and the
        attention metadata. Runs on the current (scheduler) stream."""
        plan_arrays = getattr(self.attn_backend, "plan_arrays", None)
        if plan_arrays is not None:
            plan.extra.update(plan_arrays(batch, plan.kv_lens))
        host, views = plan.pack()
        if self.is_cuda:
            dev_buf = host.pin_memory().to(self.device, non_blocking=True)
            COUNTERS.h2d_bytes += host.numel() * host.element_size()
        else:
            dev_buf = host
        dev = {k: dev_buf[s:e] for k, (s, e) in views.items()}
        batch.positions = dev["positions"]
        if self.is_cuda:
            # one launch: page-table writes, then out_loc = page_table[tok_rows, positions]
            batch.out_loc = torch.empty(dev["positions"].numel(), dtype=torch.int32, device=self.device)
            _cuda().plan_apply(self.page_table, dev["pt_rows"], dev["pt_pos"], dev["pt_slots"], dev["tok_rows"],
                               dev["positions"], batch.out_loc)
        else:
            if plan.num_pt_writes:
                self.page_table[dev["pt_rows"].long(), dev["pt_pos"].long()] = dev["pt_slots"]
            batch.out_loc = self.page_table[dev["tok_rows"].long(), dev["positions"].long()]
        meta = {"dev": dev, "max_q_len": plan.max_q_len, "max_kv_len": plan.max_kv_len}
        self.attn_backend.prepare_metadata(batch, meta)
        return dev

    def forward_batch(self, batch: Batch, args: BatchSamplingArgs, dev: dict) -> ForwardOutput:
        if batch.is_prefill:
            batch.input_ids = dev["input_ids"]
        elif self.is_cuda:
            batch.input_ids = torch.empty(dev["req_rows"].numel(), dtype=torch.int32, device=self.device)
            _cuda().gather_i32(batch.input_ids, self.last_tokens, dev["req_rows"])
        else:
            batch.input_ids = self.last_tokens[dev["req_rows"].long()]
        fused_greedy = self._fused_greedy and args.temperatures is None
        with self.ctx.forward_batch(batch):
            if self.graph_runner.can_use_cuda_graph(batch):
                out = self.graph_runner.replay(batch)
            else:
                out = self.model.forward_hidden() if self._split_lm_head else self.model.forward()
            if fused_greedy:
                ids, vals = self.model.lm_head.greedy(out[: batch.size] if batch.is_decode else out)
            elif self._split_lm_head:
                logits = self.model.lm_head.forward(out)
            else:
                logits = out
        for req in batch.reqs:
            req.complete_one()
        if fused_greedy:
            if self._lm_shard is not None:  # every rank's (best logit, id) pair per row -> the best
                shard, tp, comm = self._lm_shard
                next_tokens = self.sampler.combine_pairs(vals, ids, batch.size, tp, comm)
            else:
                next_tokens = ids
        elif self._lm_shard is not None:
            shard, tp, comm = self._lm_shard
            next_tokens = self.sampler.sample_sharded(logits[: batch.size], args, shard, tp, comm)
        else:
            next_tokens = self.sampler.sample(logits[: batch.size], args)
        next_tokens = next_tokens.to(torch.int32)
        if self.is_cuda:
            _cuda().scatter_i32(self.last_tokens, dev["sample_rows"], next_tokens.contiguous())
        else:
            self.last_tokens[dev["sample_rows"].long()] = next_tokens
        if self.is_cuda:
            cpu = torch.empty(next_tokens.shape, dtype=torch.int32, pin_memory=True)
            cpu.copy_(next_tokens, non_blocking=True)
            COUNTERS.d2h_bytes += cpu.numel() * cpu.element_size()
            ev = torch.cuda.Event()
            ev.record(self.stream)
        else:
            cpu, ev = next_tokens.clone(), _HostEvent()
        return ForwardOutput(next_tokens, cpu, ev)

    def shutdown(self) -> None:
        self.graph_runner.destroy_cuda_graphs()
        if self.is_cuda:
            torch.cuda.synchronize(self.device)
        destroy_distributed()
        if dist.is_initialized() and not self.config.external_process_group:
            dist.destroy_process_group()
        reset_global_ctx(None)
        reset_tp_info()


class BatchPlan:
    """Host-side description of one batch, packed into a single int32 upload.

    Segments: ``positions``/``tok_rows`` per token, ``input_ids`` (prefill only), page-table
    writes ``pt_rows/pt_pos/pt_slots``, per-request ``req_rows``, ``kv_lens``, ``cu_q`` and
    ``sample_rows`` (row of ``last_tokens`` that receives the sampled token).
    """

    def __init__(self, batch: Batch, pt_writes, junk_row: int):
        reqs = batch.padded_reqs
        n = len(reqs)
        cached = np.fromiter((r.cached_len for r in reqs), np.int32, n)
        self.kv_lens = np.fromiter((r.device_len for r in reqs), np.int32, n)
        self.req_rows = np.fromiter((r.table_idx for r in reqs), np.int32, n)
        ext = self.kv_lens - cached
        if batch.is_prefill:
            self.positions = np.concatenate(
                [np.arange(c, d, dtype=np.int32) for c, d in zip(cached.tolist(), self.kv_lens.tolist())]
            ) if n else np.empty(0, np.int32)
            self.tok_rows = np.repeat(self.req_rows, ext)
            self.input_ids = np.concatenate([r.input_ids[r.cached_len : r.device_len].numpy() for r in reqs])
        else:  # one token per request
            self.positions = cached
            self.tok_rows = self.req_rows
            self.input_ids = np.empty(0, np.int32)
        self.pt_rows, self.pt_pos, self.pt_slots = pt_writes
        self.num_pt_writes = len(self.pt_rows)
        self.cu_q = np.zeros(n + 1, dtype=np.int32)
        np.cumsum(ext, out=self.cu_q[1:])
        self.sample_rows = np.fromiter(
            (r.table_idx if r.max_device_len > r.device_len else junk_row for r in batch.reqs), np.int32,
            len(batch.reqs),
        )
        self.max_q_len = int(ext.max()) if n else 0
        self.max_kv_len = int(self.kv_lens.max()) if n else 0
        self.extra: Dict[str, np.ndarray] = {}  # backend-owned segments appended to the upload

    _ORDER = ("positions", "tok_rows", "input_ids", "pt_rows", "pt_pos", "pt_slots",
              "req_rows", "kv_lens", "cu_q", "sample_rows")

    def pack(self):
        parts, views, off = [], {}, 0
        for name in self._ORDER + tuple(self.extra):
            a = self.extra[name] if name in self.extra else getattr(self, name)
            n = len(a)
            views[name] = (off, off + n)
            pad = (-n) % 4  # keep every segment 16-byte aligned on the device
            parts.append(a.astype(np.int32, copy=False))
            if pad:
                parts.append(np.zeros(pad, np.int32))
            off += n + pad
        return torch.from_numpy(np.concatenate(parts)), views
