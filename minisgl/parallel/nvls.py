"""Tensor-parallel all-reduce fused with the following residual add + RMSNorm, over NVLink SHARP.

With NVLS, every rank's symmetric buffer is bound to one NVLink multicast object: a single
``multimem.ld_reduce`` on the multicast address returns the sum of all ranks' copies (the switch
does the reduction) and a single ``multimem.red`` increments a counter on every GPU. The row-
parallel ``o_proj`` / ``down_proj`` GEMMs therefore leave their partial sums unreduced, and the
RMSNorm that follows them (``post_attention_layernorm``, the next layer's ``input_layernorm``, the
final norm) runs ``nvls_allreduce_rmsnorm`` instead of all-reduce + ``fused_add_rmsnorm``: one
kernel, no second pass over the activations. Small messages use the barrier-free "LL" form
(data tagged with the call's epoch, multicast-stored into every GPU), larger ones a per-CTA barrier
plus ``multimem.ld_reduce``. The kernel is
``csrc/kernels/comm.cu`` (``nvls_ar_rmsnorm_kernel``); torch's symmetric memory only allocates the
buffer and sets up the multicast mapping.

Activations larger than the buffer (long prefill chunks) take the unfused path. This replaces the
reference's all-reduce after the row-parallel linears (python/minisgl/layers/linear.py:102-127)
plus its fused_add_rmsnorm (python/minisgl/layers/norm.py:32-38).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from minisgl._native import cuda as _cuda
from minisgl.env import ENV
from minisgl.utils import init_logger

logger = init_logger(__name__)


class NvlsNormComm:
    def __init__(self, group, cpu_group, device: torch.device, cap_bytes: int):
        import torch.distributed._symmetric_memory as symm_mem

        c = _cuda()
        self.cap = (cap_bytes + 255) // 256 * 256
        self.flag_bytes = c.nvls_flag_bytes()
        self.buf = symm_mem.empty(self.flag_bytes + 2 * self.cap, dtype=torch.uint8, device=device)
        self.hdl = symm_mem.rendezvous(self.buf, group)
        self.mc = int(self.hdl.multicast_ptr)
        if self.mc == 0:
            raise RuntimeError("symmetric memory has no multicast mapping (no NVLS on this system)")
        self.world = int(self.hdl.world_size)
        self.rank = int(self.hdl.rank)
        self.uc = int(self.hdl.buffer_ptrs[int(self.hdl.rank)])
        self.buf.zero_()
        self.state = torch.zeros(2 * c.nvls_grid(), dtype=torch.int32, device=device)
        self.timeout_ns = int(ENV.COMM_TIMEOUT_MS) * 1_000_000
        torch.cuda.synchronize(device)
        dist.barrier(group=cpu_group)

    def fits(self, x: torch.Tensor) -> bool:
        h = x.shape[-1]
        return x.dtype == torch.bfloat16 and x.numel() * 2 <= self.cap and h % 8 == 0 and h <= 16384

    def all_reduce_add_rmsnorm(self, x: torch.Tensor, residual: torch.Tensor | None, weight: torch.Tensor,
                               eps: float):
        """(sum_ranks(x) + residual) -> (rmsnorm of it, it); residual is updated in place."""
        x = x.contiguous()
        out = torch.empty_like(x)
        first = residual is None
        if first:
            residual = torch.empty_like(x)
        _cuda().nvls_allreduce_rmsnorm(self.uc, self.mc, self.rank, self.world, x, residual, weight, out, eps, self.cap,
                                       self.state, self.timeout_ns, first)
        return out, residual

    def close(self) -> None:
        self.hdl = None
        self.buf = None


def enable_nvls_norm(group, cpu_group, device: torch.device, cap_bytes: int, strict: bool = False):
    from .comm import DistributedCommunicator

    try:
        impl = NvlsNormComm(group, cpu_group, device, cap_bytes)
    except Exception as e:  # no multicast objects, no symmetric memory backend, ...
        if strict:
            raise
        logger.warning_rank0(f"NVLS fused all-reduce + RMSNorm unavailable ({e})")
        return None
    DistributedCommunicator.norm_impl = impl
    logger.info_rank0(f"NVLS fused all-reduce + RMSNorm enabled: {impl.world} ranks, {impl.cap >> 20} MiB per parity")
    return impl
