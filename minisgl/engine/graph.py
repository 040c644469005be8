"""Decode CUDA graphs (reference: python/minisgl/engine/graph.py:20-171).

One graph per padded batch size in ``[1, 2, 4, 8, 16, ..., max]`` sharing one memory pool.
Static buffers hold input ids, positions and out_loc; each graph keeps its own output: the final
normalised hidden states (the engine runs the LM head after the graph, as a greedy argmax fused into
the LM-head GEMM or as logits for sampling). Batches are padded with a dummy request whose
page-table row points at a dummy KV slot.
"""

from __future__ import annotations

import gc
from typing import Dict, List

import torch

from minisgl.core import Batch, Req, get_global_ctx
from minisgl.utils import init_logger

logger = init_logger(__name__)


def determine_graph_bs(cuda_graph_bs: List[int] | None, max_bs: int | None, free_memory: int,
                       max_running_req: int) -> List[int]:
    if cuda_graph_bs is not None:
        return sorted(cuda_graph_bs)
    if max_bs is None:
        max_bs = 256 if free_memory > 80 * (1 << 30) else 160
    max_bs = min(max_bs, max_running_req)
    if max_bs < 1:
        return []
    sizes = [b for b in (1, 2, 4) if b <= max_bs] + list(range(8, max_bs + 1, 8))
    if sizes[-1] != max_bs:
        sizes.append(max_bs)
    return sizes


class GraphRunner:
    def __init__(self, engine, graph_bs: List[int], dummy_req: Req):
        self.engine = engine
        self.graph_bs_list = sorted(graph_bs)
        self.max_graph_bs = max(graph_bs) if graph_bs else 0
        self.dummy_req = dummy_req
        self.graph_map: Dict[int, torch.cuda.CUDAGraph] = {}
        self.graph_launches: Dict[int, int] = {}
        self.outputs: Dict[int, torch.Tensor] = {}  # each graph's own output tensor (no copy-out)
        if self.max_graph_bs and engine.device.type == "cuda":
            self._capture()
        else:
            self.max_graph_bs = 0

    def _capture(self) -> None:
        eng = self.engine
        dev = eng.device
        mx = self.max_graph_bs
        eng.attn_backend.init_capture_graph(eng.aligned_max_seq_len, self.graph_bs_list)
        self.input_ids = torch.zeros(mx, dtype=torch.int32, device=dev)
        self.positions = torch.zeros(mx, dtype=torch.int32, device=dev)
        self.out_loc = torch.full((mx,), eng.dummy_slot, dtype=torch.int32, device=dev)
        torch.cuda.synchronize(dev)
        free0 = torch.cuda.mem_get_info(dev)[0]
        logger.info_rank0(f"Capturing CUDA graphs for bs={self.graph_bs_list}")
        pool = None
        ctx = get_global_ctx()
        for bs in reversed(self.graph_bs_list):
            batch = Batch(reqs=[self.dummy_req] * bs, phase="decode")
            batch.padded_reqs = batch.reqs
            eng.attn_backend.prepare_for_capture(batch)
            batch.input_ids = self.input_ids[:bs]
            batch.positions = self.positions[:bs]
            batch.out_loc = self.out_loc[:bs]
            g = torch.cuda.CUDAGraph()
            from .counters import COUNTERS

            fwd = eng.model.forward_hidden if eng._split_lm_head else eng.model.forward
            with ctx.forward_batch(batch):
                fwd()  # warm up outside the capture
                before = COUNTERS.launches
                with torch.cuda.graph(g, pool=pool, stream=eng.stream):
                    self.outputs[bs] = fwd()
                self.graph_launches[bs] = COUNTERS.launches - before
            pool = pool or g.pool()
            self.graph_map[bs] = g
        torch.cuda.synchronize(dev)
        used = free0 - torch.cuda.mem_get_info(dev)[0]
        logger.info_rank0(f"CUDA graphs captured, {used / (1 << 30):.2f} GiB")

    def can_use_cuda_graph(self, batch: Batch) -> bool:
        return batch.is_decode and 0 < batch.size <= self.max_graph_bs

    def pad_batch(self, batch: Batch) -> None:
        if self.can_use_cuda_graph(batch):
            padded = next(b for b in self.graph_bs_list if b >= batch.size)
        else:
            padded = batch.size
        batch.padded_reqs = batch.reqs + [self.dummy_req] * (padded - batch.size)

    def replay(self, batch: Batch) -> torch.Tensor:
        bs = batch.padded_size
        self.input_ids[:bs].copy_(batch.input_ids)
        self.positions[:bs].copy_(batch.positions)
        self.out_loc[:bs].copy_(batch.out_loc)
        self.engine.attn_backend.prepare_for_replay(batch)
        self.graph_map[bs].replay()
        from .counters import COUNTERS

        COUNTERS.launches += self.graph_launches[bs]
        # The graphs share one memory pool, so this tensor may alias another graph's buffers: it is
        # consumed (sampled) on the same stream before the next replay.
        return self.outputs[bs][: batch.size]

    def destroy_cuda_graphs(self) -> None:
        self.graph_map.clear()
        self.outputs.clear()
        gc.collect()
