"""Tensor-parallel all-reduce fused with the following residual add + RMSNorm, over NVLink SHARP,
and fused with the row-parallel GEMM that produces its input.

With NVLS, every rank's symmetric buffer is bound to one NVLink multicast object: a single
``multimem.ld_reduce`` on the multicast address returns the sum of all ranks' copies (the switch
does the reduction), ``multimem.st`` writes every GPU's copy and ``multimem.red`` increments a
counter on every GPU. The row-parallel ``o_proj`` / ``down_proj`` GEMMs, the vocab-parallel
embedding and the MoE combine therefore leave their partial sums unreduced, and the RMSNorm that
follows each of them (``post_attention_layernorm``, the next layer's ``input_layernorm``, the
final norm) runs ``nvls_allreduce_rmsnorm`` instead of all-reduce + ``fused_add_rmsnorm``.

Two forms (kernel: ``csrc/kernels/comm.cu``, ``nvls_ar_rmsnorm_kernel``):

* LL (small batches): each rank multicasts its partial rows tagged with the call's epoch and sums
  every rank's copy locally; no barrier; the residual stays complete on every rank.
* RS (the rest): reduce-scatter by row through ``multimem.ld_reduce``, residual add + RMSNorm of
  this rank's rows, all-gather of the normalised rows with ``multimem.st`` into the buffer's gather
  region, which is returned as the activations (a view: it is overwritten by the next RS call, by
  which time its consumer, the next column-parallel GEMM, has run). The row-parallel GEMM writes its
  output straight into this rank's staging region and its last CTA signals arrival
  (``linear_into_staging``), so the partial sum never makes a second trip through HBM and the
  collective starts the moment the GEMM's tiles land. In this form the residual stream is sharded by
  row: rank r keeps rows i with i % world == r up to date, which is all the fused norms (its only
  readers) need.

Which form runs depends only on the batch's token count, so every norm of one forward uses the same
one. Activations larger than the buffer (long prefill chunks) take the unfused path. This replaces
the reference's all-reduce after the row-parallel linears (python/minisgl/layers/linear.py:102-127)
plus its fused_add_rmsnorm (python/minisgl/layers/norm.py:32-38).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from minisgl._native import cuda as _cuda
from minisgl.env import ENV
from minisgl.utils import init_logger

logger = init_logger(__name__)

MODE_LL, MODE_STAGE, MODE_PRESTAGED, MODE_GEMM_ARRIVED = 0, 1, 2, 3


class NvlsNormComm:
    def __init__(self, group, cpu_group, device: torch.device, cap_bytes: int):
        import torch.distributed._symmetric_memory as symm_mem

        c = _cuda()
        self.cap = (cap_bytes + 255) // 256 * 256
        self.flag_bytes = c.nvls_flag_bytes()
        # [flags | LL parity 0 | LL parity 1 | RS staging | RS gather]
        self.buf = symm_mem.empty(self.flag_bytes + 4 * self.cap, dtype=torch.uint8, device=device)
        self.hdl = symm_mem.rendezvous(self.buf, group)
        self.mc = int(self.hdl.multicast_ptr)
        if self.mc == 0:
            raise RuntimeError("symmetric memory has no multicast mapping (no NVLS on this system)")
        self.world = int(self.hdl.world_size)
        self.rank = int(self.hdl.rank)
        self.uc = int(self.hdl.buffer_ptrs[int(self.hdl.rank)])
        self.buf.zero_()
        self.state = torch.zeros(c.nvls_state_words(), dtype=torch.int32, device=device)
        self.ticket = self.state.data_ptr() + c.nvls_ticket_offset()
        self.timeout_ns = int(ENV.COMM_TIMEOUT_MS) * 1_000_000
        self.ll_limit = int(ENV.NVLS_LL_BYTES)
        self.gemm_fusion = bool(ENV.NVLS_GEMM_FUSION)
        self._staged_by_gemm = None  # data_ptr of the staging view the last fused GEMM wrote
        torch.cuda.synchronize(device)
        dist.barrier(group=cpu_group)

    # ------------------------------------------------------------------ shapes and regions
    def fits(self, x: torch.Tensor) -> bool:
        h = x.shape[-1]
        if not (x.dtype == torch.bfloat16 and x.numel() * 2 <= self.cap and h % 8 == 0 and h <= 16384):
            return False
        return self.is_ll(x.numel() // h, h) or h <= 8192  # the RS form takes hidden sizes up to 8192

    def is_ll(self, tokens: int, hidden: int) -> bool:
        b = self.world * tokens * hidden * 4
        return b <= self.cap and b <= self.ll_limit

    def _region(self, index: int, tokens: int, hidden: int) -> torch.Tensor:
        off = self.flag_bytes + index * self.cap
        return self.buf[off : off + tokens * hidden * 2].view(torch.bfloat16).view(tokens, hidden)

    def staging(self, tokens: int, hidden: int) -> torch.Tensor:
        return self._region(2, tokens, hidden)

    def gather(self, tokens: int, hidden: int) -> torch.Tensor:
        return self._region(3, tokens, hidden)

    # ------------------------------------------------------------------ fused paths
    def linear_into_staging(self, x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None):
        """Row-parallel GEMM fused with the collective's first phase: ``x @ weight^T (+ bias)`` is
        written into this rank's staging region and the GEMM's last CTA signals arrival to every
        rank. Returns the staging view (pass it to ``all_reduce_add_rmsnorm``), or None when this
        batch uses the LL form or does not fit (the caller then runs the plain GEMM)."""
        tokens, hidden = x.shape[0], weight.shape[0]
        if (not self.gemm_fusion or tokens == 0 or weight.dim() != 2 or hidden % 8 != 0 or hidden > 8192
                or tokens * hidden * 2 > self.cap or self.is_ll(tokens, hidden)):
            return None
        y = self.staging(tokens, hidden)
        _cuda().gemm_signal(y, x.contiguous(), weight, bias, self.ticket, self.mc)
        self._staged_by_gemm = y.data_ptr()
        return y

    def all_reduce_add_rmsnorm(self, x: torch.Tensor, residual: torch.Tensor | None, weight: torch.Tensor,
                               eps: float, trace: torch.Tensor | None = None):
        """(sum_ranks(x) + residual) -> (rmsnorm of it, it); residual is updated in place (RS form:
        this rank's rows only)."""
        x = x.contiguous()
        tokens, hidden = x.numel() // x.shape[-1], x.shape[-1]
        first = residual is None
        if first:
            residual = torch.empty_like(x)
        if self.is_ll(tokens, hidden):
            mode, out = MODE_LL, torch.empty_like(x)
        else:
            out = self.gather(tokens, hidden).view(x.shape)
            mode = MODE_GEMM_ARRIVED if self._staged_by_gemm == x.data_ptr() else MODE_STAGE
        self._staged_by_gemm = None
        _cuda().nvls_allreduce_rmsnorm(self.uc, self.mc, self.rank, self.world, x, residual, weight, out, eps,
                                       self.cap, self.state, self.timeout_ns, first, mode, trace)
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
    logger.info_rank0(f"NVLS fused all-reduce + RMSNorm enabled: {impl.world} ranks, {impl.cap >> 20} MiB regions")
    return impl
