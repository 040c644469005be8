from __future__ import annotations

import torch

from minisgl.layers.base import BaseOP


class BaseLLMModel(BaseOP):
    """A causal LM: ``forward()`` reads the active batch from the global context and returns
    logits ``[batch.size, vocab]`` (reference: python/minisgl/models/base.py:12-14)."""

    def forward(self) -> torch.Tensor:
        raise NotImplementedError
