"""This engine's tensor-parallel collectives over CUDA IPC peer memory (NVLink / NVSwitch).

Each rank allocates one symmetric buffer (``[flags | data parity 0 | data parity 1]``), exports it
with a CUDA IPC handle, and maps every peer's buffer. The kernels in ``csrc/kernels/comm.cu``
synchronize with per-CTA epoch flags (bounded waits) and read peers' data directly:

* all-reduce: one-shot (every rank sums all copies) up to ``ONE_SHOT_MAX`` bytes, two-shot
  (reduce-scatter + all-gather through peer memory) above;
* all-gather along dim 0.

Messages larger than the buffer go to the NCCL baseline (``TorchDistributedImpl``). This replaces
the reference's NCCL symmetric-window wrapper (python/minisgl/kernel/csrc/src/pynccl.cu).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from minisgl._native import cuda as _cuda
from minisgl.env import ENV
from minisgl.utils import init_logger

from .comm import CommImpl, DistributedCommunicator

logger = init_logger(__name__)

ONE_SHOT_MAX = 256 * 1024


class PeerCommImpl(CommImpl):
    def __init__(self, cpu_group, device: torch.device, max_bytes: int, fallback: CommImpl):
        c = _cuda()
        self.rank = dist.get_rank(cpu_group)
        self.world = dist.get_world_size(cpu_group)
        if self.world > 8:
            raise ValueError("peer collectives support up to 8 ranks")
        self.device = device
        self.cap = (max_bytes + 15) // 16 * 16
        self.flag_bytes = c.peer_flag_bytes()
        self.ptr = c.peer_alloc(self.flag_bytes + 2 * self.cap)
        handles = [None] * self.world
        dist.all_gather_object(handles, c.ipc_handle(self.ptr), group=cpu_group)
        self.bases = [self.ptr if r == self.rank else c.ipc_open(h) for r, h in enumerate(handles)]
        self.state = torch.zeros(2 * c.peer_grid(), dtype=torch.int32, device=device)
        self.timeout_ns = int(ENV.COMM_TIMEOUT_MS) * 1_000_000
        self.fallback = fallback
        self._closed = False
        dist.barrier(group=cpu_group)

    def _run(self, mode: int, out: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
        _cuda().peer_collective(mode, out, x, self.bases, self.rank, self.cap, self.state, self.timeout_ns)
        return out

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        nbytes = x.numel() * x.element_size()
        if x.dtype != torch.bfloat16 or nbytes > self.cap or nbytes % 16:
            return self.fallback.all_reduce(x)
        x = x.contiguous()
        return self._run(0 if nbytes <= ONE_SHOT_MAX else 1, torch.empty_like(x), x)

    def all_gather(self, x: torch.Tensor) -> torch.Tensor:
        x = x.contiguous()
        nbytes = x.numel() * x.element_size()
        if nbytes > self.cap or nbytes % 16:
            return self.fallback.all_gather(x)
        out = torch.empty((self.world * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
        return self._run(2, out, x)

    def close(self) -> None:
        if self._closed:
            return
        self._closed = True
        c = _cuda()
        torch.cuda.synchronize(self.device)
        for r, b in enumerate(self.bases):
            if r != self.rank:
                c.ipc_close(b)
        c.peer_free(self.ptr)


def enable_peer_comm(cpu_group, device: torch.device, max_bytes: int, strict: bool = False) -> PeerCommImpl | None:
    """Push the peer-memory implementation on the communicator stack (NCCL stays the fallback)."""
    fallback = DistributedCommunicator.active()
    try:
        impl = PeerCommImpl(cpu_group, device, max_bytes, fallback)
    except Exception as e:  # no P2P between these devices, IPC unavailable, ...
        if strict:
            raise
        logger.warning_rank0(f"peer collectives unavailable ({e}); using NCCL")
        return None
    DistributedCommunicator.push(impl)
    logger.info_rank0(f"peer collectives enabled: {impl.world} ranks, {impl.cap >> 20} MiB buffer")
    return impl
