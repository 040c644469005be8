"""Vocab-parallel embedding and LM head (reference: python/minisgl/layers/embedding.py:14-110).

Each rank owns ``ceil(V / tp)`` consecutive vocab rows. The embedding gathers owned rows (zeros
elsewhere) and sums over ranks; the LM head computes local logits for the last token of each
request and gathers them over ranks.
"""

from __future__ import annotations

from typing import Dict

import torch

from minisgl import ops
from minisgl.core import get_global_ctx
from minisgl.parallel import DistributedCommunicator, get_tp_info
from minisgl.utils import div_ceil, nvtx_annotate

from .base import BaseOP


class VocabParallelEmbedding(BaseOP):
    def __init__(self, num_embeddings: int, embedding_dim: int):
        info = get_tp_info()
        self._tp = info.size
        self.num_embeddings = num_embeddings
        self.num_embeddings_tp = div_ceil(num_embeddings, info.size)
        start = self.num_embeddings_tp * info.rank
        stop = min(start + self.num_embeddings_tp, num_embeddings)
        self._vocab_range = (start, stop - start)
        self.weight = torch.empty(self.num_embeddings_tp, embedding_dim)
        self._comm = DistributedCommunicator()

    def named_children(self):
        for k, v in super().named_children():
            if k not in ("num_embeddings", "num_embeddings_tp"):
                yield k, v

    # set by the model when the first layer's input norm can take the unreduced per-rank rows
    # (fused all-reduce + RMSNorm); `deferred` tells whether the last forward left them unreduced
    defer_to_norm = False
    deferred = False

    @nvtx_annotate("Embedding")
    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        if self._tp == 1:
            return ops.embedding(self.weight, ids)
        y = ops.embedding(self.weight, ids, *self._vocab_range)
        fused = DistributedCommunicator.norm_impl
        self.deferred = self.defer_to_norm and fused is not None and fused.fits(y)
        return y if self.deferred else self._comm.all_reduce(y)


class ParallelLMHead(VocabParallelEmbedding):
    def __init__(self, num_embeddings: int, embedding_dim: int, bias: bool = False,
                 tie_word_embeddings: bool = False, tied_embedding: VocabParallelEmbedding | None = None):
        super().__init__(num_embeddings, embedding_dim)
        self.bias = torch.empty(self.num_embeddings_tp) if bias else None
        self._tied = tied_embedding
        if (tied_embedding is not None) != tie_word_embeddings:
            raise ValueError("tied_embedding must be given iff tie_word_embeddings")
        if tied_embedding is not None:
            del self.weight

    def load_state_dict(self, state_dict: Dict[str, torch.Tensor], *, prefix: str = "", _internal: bool = False) -> None:
        if self._tied is None:
            return super().load_state_dict(state_dict, prefix=prefix, _internal=_internal)
        state_dict.pop(f"{prefix}.weight", None)
        state_dict.pop(f"{prefix}.bias", None)

    def state_dict(self, *, prefix: str = "", result=None):
        if self._tied is None:
            return super().state_dict(prefix=prefix, result=result)
        return {} if result is None else result

    @property
    def lm_weight(self) -> torch.Tensor:
        return self._tied.weight if self._tied is not None else self.weight

    # At TP > 1 the engine sets this: forward returns this rank's vocab shard and the sampler
    # combines shards (greedy: per-rank (max, argmax) pairs instead of gathering all logits).
    return_local = False

    @property
    def vocab_shard(self) -> tuple:
        """(first vocab id of this rank's shard, number of valid ids in it)."""
        return self._vocab_range

    @nvtx_annotate("LMHead")
    def greedy(self, x: torch.Tensor):
        """Greedy pick of this rank's vocabulary shard without writing the logits: the argmax is
        taken inside the LM-head GEMM's epilogue. Returns (global token id int32, its logit fp32)
        per row; at TP > 1 the sampler combines the ranks' pairs."""
        batch = get_global_ctx().batch
        if batch.is_prefill:
            x = x.index_select(0, batch.attn_metadata.get_last_indices(batch.size))
        start, valid = self._vocab_range
        return ops.lm_head_argmax(x, self.lm_weight, self.bias, valid, start)

    @nvtx_annotate("LMHead")
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        batch = get_global_ctx().batch
        if batch.is_prefill:
            x = x.index_select(0, batch.attn_metadata.get_last_indices(batch.size))
        logits = ops.linear(x, self.lm_weight, self.bias)
        if self._tp == 1 or self.return_local:
            return logits
        rows, vl = logits.shape
        full = self._comm.all_gather(logits)  # [tp * rows, V/tp]
        full = full.view(self._tp, rows, vl).permute(1, 0, 2).reshape(rows, self._tp * vl)
        return full[:, : self.num_embeddings]
