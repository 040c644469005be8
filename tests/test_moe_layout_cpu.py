"""Expert weight layout for the gated grouped GEMM (CPU): interleaving gate / up rows in 128-row
blocks and padding the intermediate size to a whole block keeps every expert's product unchanged."""

import pytest
import torch

from minisgl.ops.moe import interleave_experts
from minisgl.ops.reference import GATE_UP_BLOCK, deinterleave_gate_up


@pytest.mark.parametrize("inter", [128, 360, 384, 2880])
def test_interleave_experts_preserves_the_mlp(inter):
    g = torch.Generator().manual_seed(inter)
    E, H = 3, 64
    w1 = torch.randn(E, 2 * inter, H, generator=g)
    w2 = torch.randn(E, H, inter, generator=g)
    b1 = torch.randn(E, 2 * inter, generator=g)
    w1i, w2i, b1i = interleave_experts(w1, w2, b1)
    ip = -(-inter // GATE_UP_BLOCK) * GATE_UP_BLOCK
    assert w1i.shape == (E, 2 * ip, H) and w2i.shape == (E, H, ip) and b1i.shape == (E, 2 * ip)
    x = torch.randn(5, H, generator=g)
    for e in range(E):
        gate, up = (x @ w1[e].t() + b1[e]).chunk(2, dim=-1)
        ref = (torch.nn.functional.silu(gate) * up) @ w2[e].t()
        gi, ui = deinterleave_gate_up(x @ w1i[e].t() + b1i[e])
        assert torch.equal(gi[:, inter:], torch.zeros_like(gi[:, inter:]))  # padding rows produce 0
        out = (torch.nn.functional.silu(gi) * ui) @ w2i[e].t()
        torch.testing.assert_close(out, ref, rtol=1e-4, atol=5e-3)  # fp32 summation order
