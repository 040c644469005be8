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


def _random_mxfp4(E, n, k, seed):
    g = torch.Generator().manual_seed(seed)
    blocks = torch.randint(0, 256, (E, n, k // 32, 16), generator=g, dtype=torch.int32).to(torch.uint8)
    scales = torch.randint(118, 130, (E, n, k // 32), generator=g, dtype=torch.int32).to(torch.uint8)
    return blocks, scales


@pytest.mark.parametrize("n,k,tile", [(256, 128, 256), (200, 192, 128), (2880, 2880, 128)])
def test_mxfp4_pack_round_trips(n, k, tile):
    """The k-block-major fp4 layout of the grouped GEMM encodes exactly the dequantised weights;
    padding rows decode to zero."""
    from minisgl.moe.mxfp4 import Mxfp4Experts, dequant_mxfp4

    blocks, scales = _random_mxfp4(2, n, k, n + k)
    packed = Mxfp4Experts.pack(blocks, scales, tile)
    assert packed.shape == (2, n, k) and packed.q.shape[2] % tile == 0
    assert packed.q.shape == (2, k // 64, packed.q.shape[2], 32) and packed.s.shape[-1] == 2
    assert torch.equal(packed.dequant(torch.float32), dequant_mxfp4(blocks, scales, torch.float32))
    assert not packed.q[:, :, n:].any() and not packed.s[:, :, n:].any()


@pytest.mark.parametrize("inter", [128, 360, 2880])
def test_mxfp4_interleave_matches_the_bf16_layout(inter):
    """Interleaving MXFP4 blocks / scales by rows (and padding the down projection's input dim)
    gives the bf16 ``interleave_experts`` layout of the dequantised weights."""
    from minisgl.moe.mxfp4 import dequant_mxfp4, interleave_rows, pad_k

    E, H = 2, 64
    b1, s1 = _random_mxfp4(E, 2 * inter, H, inter)
    b2, s2 = _random_mxfp4(E, H, -(-inter // 32) * 32, inter + 1)
    if inter % 32:
        return  # the down projection's input dim must be whole 32-value blocks
    w1, w2 = dequant_mxfp4(b1, s1, torch.float32), dequant_mxfp4(b2, s2, torch.float32)
    w1i, w2i, _ = interleave_experts(w1, w2, None)
    assert torch.equal(dequant_mxfp4(interleave_rows(b1), interleave_rows(s1), torch.float32), w1i)
    ip = w1i.shape[1] // 2
    assert torch.equal(dequant_mxfp4(*pad_k(b2, s2, ip), torch.float32), w2i)


def test_moe_layer_dequantises_mxfp4_off_the_gpu():
    """On the CPU the MoE layer turns ``<proj>_blocks`` / ``_scales`` into the bf16 weights."""
    from minisgl.layers.moe import MoELayer
    from minisgl.moe.mxfp4 import dequant_mxfp4
    from minisgl.parallel import set_tp_info
    from minisgl.parallel.info import reset_tp_info

    set_tp_info(0, 1)
    try:
        layer = MoELayer(4, 2, 64, 128, activation="swiglu_oai", has_bias=True)
        b1, s1 = _random_mxfp4(4, 256, 64, 1)
        b2, s2 = _random_mxfp4(4, 64, 128, 2)
        sd = {"gate_up_proj_blocks": b1, "gate_up_proj_scales": s1, "down_proj_blocks": b2,
              "down_proj_scales": s2, "gate_up_proj_bias": torch.zeros(4, 256), "down_proj_bias": torch.zeros(4, 64)}
        layer.load_state_dict(sd)
    finally:
        reset_tp_info()
    assert torch.equal(layer.gate_up_proj, dequant_mxfp4(b1, s1, torch.float32))
    assert torch.equal(layer.down_proj, dequant_mxfp4(b2, s2, torch.float32))
