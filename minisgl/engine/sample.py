"""Sampling (reference: python/minisgl/engine/sample.py:13-75).

Greedy batches run the row argmax kernel. Otherwise one kernel applies temperature, top-k and
top-p and draws with the Gumbel-max trick from counter-based noise keyed by
``(seed, step, token id)``: a request's draw does not depend on its batch neighbours or on the TP
degree.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import List

import torch

from minisgl import ops
from minisgl.utils import nvtx_annotate


# Largest top-k served from per-shard candidate lists under vocabulary parallelism
SHARD_CANDIDATES_MAX = 1024
# Extra candidates per shard beyond the largest top-k, for tokens tied at the k-th value
SHARD_CANDIDATE_SLACK = 16


@dataclass
class BatchSamplingArgs:
    temperatures: torch.Tensor | None
    top_k: torch.Tensor | None = None
    top_p: torch.Tensor | None = None
    seeds: torch.Tensor | None = None
    steps: torch.Tensor | None = None
    # how vocabulary shards combine (host-side summary of the batch's parameters):
    # "temperature": no row uses top-k or top-p; "topk": every sampled row has top-k <= `cand`;
    # "full": anything else
    mode: str = "full"
    cand: int = 0


def _to_device(data: List, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    t = torch.tensor(data, dtype=dtype)
    if device.type == "cuda":
        from .counters import COUNTERS

        COUNTERS.h2d_bytes += t.numel() * t.element_size()
        return t.pin_memory().to(device, non_blocking=True)
    return t


@dataclass
class Sampler:
    device: torch.device
    vocab_size: int

    def prepare(self, batch) -> BatchSamplingArgs:
        if all(r.greedy for r in batch.reqs):
            return BatchSamplingArgs(temperatures=None)
        params = [r.sampling_params for r in batch.reqs]
        temps = [0.0 if p.is_greedy else max(p.temperature, 1e-6) for p in params]
        ks = [min(p.top_k, self.vocab_size) if p.top_k >= 1 else self.vocab_size for p in params]
        ps = [min(max(p.top_p, 1e-6), 1.0) for p in params]
        sampled = [i for i, t in enumerate(temps) if t > 0]
        mode, cand = "full", 0
        if all(ks[i] >= self.vocab_size and ps[i] >= 1.0 for i in sampled):
            mode = "temperature"
        elif all(ks[i] < self.vocab_size and ks[i] <= SHARD_CANDIDATES_MAX for i in sampled):
            mode, cand = "topk", max(ks[i] for i in sampled)
        seeds = [(p.seed if p.seed is not None else r.uid * 2654435761 + 12345) & 0x7FFFFFFF
                 for p, r in zip(params, batch.reqs)]
        steps = [r.device_len for r in batch.reqs]
        d = self.device
        return BatchSamplingArgs(
            temperatures=_to_device(temps, torch.float32, d),
            top_k=_to_device(ks, torch.int32, d),
            top_p=_to_device(ps, torch.float32, d),
            seeds=_to_device(seeds, torch.int64, d),
            steps=_to_device(steps, torch.int64, d),
            mode=mode,
            cand=cand,
        )

    @nvtx_annotate("Sampler")
    def sample(self, logits: torch.Tensor, args: BatchSamplingArgs) -> torch.Tensor:
        if args.temperatures is None:
            return ops.argmax(logits)
        return ops.sample(logits, args.temperatures, args.top_k, args.top_p, args.seeds, args.steps)

    def sample_sharded(self, local: torch.Tensor, args: BatchSamplingArgs, shard: tuple, tp: int,
                       comm) -> torch.Tensor:
        """``local``: this rank's logits for vocab ids [start, start + valid) (row stride = the
        padded shard width). Greedy batches exchange one (max, global argmax) pair per row and
        rank instead of the logits (the reference gathers all of them,
        python/minisgl/layers/embedding.py:87-110); ties resolve to the lowest id as in the
        unsharded argmax.

        Sampled batches use the Gumbel-max draw, whose noise is keyed by the global token id, so
        shards reproduce the unsharded draw: with temperature only, each rank draws over its
        shard and the ranks exchange (winning score, id) pairs like the greedy path; with top-k
        <= SHARD_CANDIDATES_MAX on every sampled row, each rank contributes its top-(k + slack)
        logits, the candidate lists are gathered ([rows, tp * (k + slack)] instead of
        [rows, vocab]) and the kernel samples over them with their token ids (top-k and the top-p
        nucleus of the top-k set lie inside the union; exact unless more than the slack of one
        shard's tokens tie at the k-th value). Other batches gather the full logits."""
        start, valid = shard
        rows, width = local.shape
        if args.temperatures is None:
            idx, val = ops.argmax(local, vocab=valid, with_values=True)
            return self._combine_pairs(val, idx + start, rows, tp, comm)
        if args.mode == "temperature":
            ids, val = ops.sample(local[:, :valid], args.temperatures, args.top_k, args.top_p, args.seeds, args.steps,
                                  id_offset=start, with_values=True)
            return self._combine_pairs(val, ids, rows, tp, comm)
        if args.mode == "topk":
            c = min(args.cand + SHARD_CANDIDATE_SLACK, valid)
            val, idx = torch.topk(local[:, :valid].float(), c, dim=1)
            pack = torch.stack([val, (idx.to(torch.int32) + start).view(torch.float32)], dim=2)  # [rows, c, 2]
            allp = comm.all_gather(pack.contiguous()).view(tp, rows, c, 2).permute(1, 0, 2, 3).reshape(rows, tp * c, 2)
            cid = allp[:, :, 1].contiguous().view(torch.int32)
            cid, order = torch.sort(cid, dim=1)  # ascending ids: column ties resolve to the lowest id
            cval = allp[:, :, 0].gather(1, order).contiguous()
            return ops.sample(cval, args.temperatures, args.top_k, args.top_p, args.seeds, args.steps,
                              col_ids=cid.contiguous())
        full = comm.all_gather(local.contiguous()).view(tp, rows, width).permute(1, 0, 2).reshape(rows, tp * width)
        return self.sample(full[:, : self.vocab_size], args)

    @nvtx_annotate("Sampler")
    def combine_pairs(self, val: torch.Tensor, ids: torch.Tensor, rows: int, tp: int, comm) -> torch.Tensor:
        """Greedy picks made per vocabulary shard (in the LM-head GEMM) -> the batch's tokens."""
        return self._combine_pairs(val, ids, rows, tp, comm)

    @staticmethod
    def _combine_pairs(val: torch.Tensor, ids: torch.Tensor, rows: int, tp: int, comm) -> torch.Tensor:
        """Each rank's (score, token id) per row -> the token of the best score; ranks hold
        ascending id ranges, so the first maximal rank is the lowest id among ties."""
        pair = torch.stack([val.float(), ids.to(torch.int32).view(torch.float32)], dim=1)  # id bit-cast into fp32
        allp = comm.all_gather(pair.contiguous()).view(tp, rows, 2)
        best = torch.argmax(allp[:, :, 0], dim=0)
        out = allp[:, :, 1].contiguous().view(torch.int32)
        return out.gather(0, best.view(1, rows)).view(rows)
