"""MXFP4 expert weights kept in HBM (gpt-oss checkpoints; OCP microscaling format): e2m1 values two
per byte (low nibble first) in blocks of 32 along the input dim, one e8m0 scale (bias 127) per block.

``Mxfp4Experts`` holds one expert projection ``[E, N, K]`` for the fp4 grouped GEMM
(``gemm_grouped_fp4``) in a k-block-major layout, so one (expert, 64-value K block, weight tile)
is a single contiguous copy of each array:

* ``q`` uint8 ``[E, K/64, Np, 32]``: e2m1 pairs, rows padded to ``Np`` (a whole number of weight tiles);
* ``s`` uint8 ``[E, K/64, Np, 2]``: the two e8m0 scales of each row's 64 values.

Row permutations (the tensor-parallel gate / up split, the 128-row gate / up interleave of the gated
GEMM, padding) act on the checkpoint's ``blocks [E, N, K/32, 16]`` and ``scales [E, N, K/32]``
before packing. The kernel converts each tile to bf16 exactly (a power-of-two scale on e2m1
values), so results equal the bf16 path run on ``dequant_mxfp4`` weights.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from minisgl.ops.reference import GATE_UP_BLOCK

# e2m1 code -> value (sign bit 3, exponent bits 2..1, mantissa bit 0)
E2M1 = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0)


def dequant_mxfp4(blocks: torch.Tensor, scales: torch.Tensor, dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """``blocks [..., G, 16]`` uint8 (32 e2m1 values per block, low nibble first), ``scales [..., G]``
    uint8 e8m0 -> ``[..., G * 32]``. Processed in chunks of rows to bound temporaries."""
    if blocks.shape[:-1] != scales.shape or blocks.shape[-1] != 16:
        raise ValueError(f"mxfp4 blocks {tuple(blocks.shape)} / scales {tuple(scales.shape)} mismatch")
    lut = torch.tensor(E2M1, dtype=torch.float32, device=blocks.device)
    G = blocks.shape[-2]
    out = torch.empty(blocks.shape[:-2] + (G * 32,), dtype=dtype, device=blocks.device)
    flat_b = blocks.reshape(-1, G, 16)
    flat_s = scales.reshape(-1, G)
    flat_o = out.view(-1, G * 32)
    step = max(1, (1 << 22) // (G * 32))  # rows per chunk: ~4M values
    for i in range(0, flat_b.shape[0], step):
        b = flat_b[i : i + step].to(torch.uint8)
        v = torch.stack([lut[(b & 0x0F).long()], lut[(b >> 4).long()]], dim=-1).reshape(b.shape[0], G, 32)
        v = torch.ldexp(v, (flat_s[i : i + step].to(torch.int32) - 127).unsqueeze(-1).to(torch.float32))
        flat_o[i : i + step] = v.reshape(b.shape[0], -1).to(dtype)
    return out


def interleave_rows(t: torch.Tensor) -> torch.Tensor:
    """``[E, 2I, ...]`` as [gate; up] halves -> gate / up rows interleaved in blocks of
    GATE_UP_BLOCK, I padded up to a whole block with zero rows (the layout ``interleave_experts``
    gives bf16 weights); works on MXFP4 blocks, scales and biases alike."""
    E, two_i = t.shape[:2]
    inter = two_i // 2
    ip = -(-inter // GATE_UP_BLOCK) * GATE_UP_BLOCK
    nb = ip // GATE_UP_BLOCK
    rest = tuple(t.shape[2:])
    out = torch.zeros((E, 2 * ip) + rest, dtype=t.dtype, device=t.device)
    v = out.view((E, nb, 2, GATE_UP_BLOCK) + rest)
    for half in range(2):
        part = torch.zeros((E, ip) + rest, dtype=t.dtype, device=t.device)
        part[:, :inter] = t[:, half * inter : (half + 1) * inter]
        v[:, :, half] = part.view((E, nb, GATE_UP_BLOCK) + rest)
    return out


def pad_k(blocks: torch.Tensor, scales: torch.Tensor, k: int):
    """Zero-pad the input dim (in 32-value blocks) up to ``k`` values."""
    g = k // 32
    if blocks.shape[2] == g:
        return blocks, scales
    pb = torch.zeros(blocks.shape[:2] + (g, 16), dtype=blocks.dtype, device=blocks.device)
    ps = torch.zeros(scales.shape[:2] + (g,), dtype=scales.dtype, device=scales.device)
    pb[:, :, : blocks.shape[2]] = blocks
    ps[:, :, : scales.shape[2]] = scales
    return pb, ps


@dataclass
class Mxfp4Experts:
    q: torch.Tensor  # uint8 [E, K/64, Np, 32]
    s: torch.Tensor  # uint8 [E, K/64, Np, 2]
    n: int           # logical rows

    @property
    def shape(self):
        return (self.q.shape[0], self.n, self.q.shape[1] * 64)

    @property
    def is_cuda(self) -> bool:
        return self.q.is_cuda

    @property
    def device(self) -> torch.device:
        return self.q.device

    @classmethod
    def pack(cls, blocks: torch.Tensor, scales: torch.Tensor, row_tile: int) -> "Mxfp4Experts":
        """``blocks [E, N, K/32, 16]``, ``scales [E, N, K/32]`` (K a multiple of 64) -> packed, rows
        padded to a multiple of ``row_tile``."""
        E, n, g = scales.shape
        if g % 2:
            raise ValueError(f"MXFP4 input dim {g * 32} is not a multiple of 64")
        npad = -(-n // row_tile) * row_tile
        q = torch.zeros(E, g // 2, npad, 32, dtype=torch.uint8, device=blocks.device)
        s = torch.zeros(E, g // 2, npad, 2, dtype=torch.uint8, device=blocks.device)
        q[:, :, :n] = blocks.reshape(E, n, g // 2, 32).permute(0, 2, 1, 3)
        s[:, :, :n] = scales.reshape(E, n, g // 2, 2).permute(0, 2, 1, 3)
        return cls(q.contiguous(), s.contiguous(), n)

    def dequant(self, dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
        """The ``[E, N, K]`` weights these bytes encode."""
        E, kb, _, _ = self.q.shape
        blocks = self.q[:, :, : self.n].permute(0, 2, 1, 3).reshape(E, self.n, kb * 2, 16)
        scales = self.s[:, :, : self.n].permute(0, 2, 1, 3).reshape(E, self.n, kb * 2)
        return dequant_mxfp4(blocks, scales, dtype)

    def nbytes(self) -> int:
        return self.q.numel() + self.s.numel()
