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
        params = [r.sampling_params for r in batch.reqs]
        if all(p.is_greedy for p in params):
            return BatchSamplingArgs(temperatures=None)
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

    def sample(self, logits: torch.Tensor, args: BatchSamplingArgs) -> torch.Tensor:
        if args.temperatures is None:
            return ops.argmax(logits)
        return ops.sample(logits, args.temperatures, args.top_k, args.top_p, args.seeds, args.steps)
