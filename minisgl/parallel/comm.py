"""Tensor-parallel collectives used by the layers.

``DistributedCommunicator`` forwards to the active implementation:

* ``TorchDistributedImpl`` - ``torch.distributed`` on the TP group (gloo on CPU, NCCL on GPU).
  This is the NCCL baseline path (reference: python/minisgl/distributed/impl.py:15-97).
* ``PeerCommImpl`` (``parallel/peer.py``) - this engine's own all-reduce / all-gather kernels over
  CUDA IPC peer memory, enabled by ``enable_peer_comm``.
"""

from __future__ import annotations

from typing import List

import torch
import torch.distributed as dist


class CommImpl:
    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        raise NotImplementedError

    def all_gather(self, x: torch.Tensor) -> torch.Tensor:
        raise NotImplementedError


class TorchDistributedImpl(CommImpl):
    def __init__(self, group=None):
        self.group = group

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        dist.all_reduce(x, op=dist.ReduceOp.SUM, group=self.group)
        return x

    def all_gather(self, x: torch.Tensor) -> torch.Tensor:
        n = dist.get_world_size(self.group)
        out = torch.empty((n * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(out, x.contiguous(), group=self.group)
        return out


class DistributedCommunicator:
    _stack: List[CommImpl] = [TorchDistributedImpl()]
    # fused all-reduce + residual add + RMSNorm (NVLS), used by the norms that follow row-parallel
    # linears; None when unavailable
    norm_impl = None

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        return self._stack[-1].all_reduce(x)

    def all_gather(self, x: torch.Tensor) -> torch.Tensor:
        return self._stack[-1].all_gather(x)

    @classmethod
    def push(cls, impl: CommImpl) -> None:
        cls._stack.append(impl)

    @classmethod
    def reset(cls) -> None:
        cls._stack = [TorchDistributedImpl()]
        cls.norm_impl = None

    @classmethod
    def active(cls) -> CommImpl:
        return cls._stack[-1]


def set_torch_group(group) -> None:
    DistributedCommunicator._stack[0] = TorchDistributedImpl(group)


def destroy_distributed() -> None:
    for impl in DistributedCommunicator._stack + [DistributedCommunicator.norm_impl]:
        close = getattr(impl, "close", None)
        if close is not None:
            close()
    DistributedCommunicator.reset()
