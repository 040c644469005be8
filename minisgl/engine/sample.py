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


@dataclass
class BatchSamplingArgs:
    temperatures: torch.Tensor | None
    top_k: torch.Tensor | None = None
    top_p: torch.Tensor | None = None
    seeds: torch.Tensor | None = None
    steps: torch.Tensor | None = None


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
        ks = [p.top_k if p.top_k >= 1 else self.vocab_size for p in params]
        ps = [min(max(p.top_p, 1e-6), 1.0) for p in params]
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
        unsharded argmax. Other batches gather the full logits and run the sampling kernel."""
        start, valid = shard
        rows, width = local.shape
        if args.temperatures is None:
            idx, val = ops.argmax(local, vocab=valid, with_values=True)
            pair = torch.stack([val, (idx + start).view(torch.float32)], dim=1)  # id bit-cast into fp32
            allp = comm.all_gather(pair.contiguous()).view(tp, rows, 2)
            best = torch.argmax(allp[:, :, 0], dim=0)  # first maximal rank = lowest id among ties
            ids = allp[:, :, 1].contiguous().view(torch.int32)
            return ids.gather(0, best.view(1, rows)).view(rows)
        full = comm.all_gather(local.contiguous()).view(tp, rows, width).permute(1, 0, 2).reshape(rows, tp * width)
        return self.sample(full[:, : self.vocab_size], args)
