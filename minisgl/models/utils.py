"""Shared decoder blocks (reference: python/minisgl/models/utils.py:25-123).

``GatedMLP``: gate_up (column parallel, gate/up interleaved in 64-row blocks so the GEMM epilogue
applies the activation) -> down (row parallel + reduce).
``MoEMLP``: replicated router + ``MoELayer``.
``RopeAttn``: merged qkv -> fused QK-norm/RoPE/KV-store -> paged attention -> o_proj.
"""

from __future__ import annotations

from typing import Tuple

import torch

from minisgl import ops
from minisgl.layers import (
    AttentionLayer,
    LinearColParallelMerged,
    LinearOProj,
    LinearQKVMerged,
    LinearReplicated,
    LinearRowParallel,
    MoELayer,
    OPList,
    ParallelLMHead,
    RMSNorm,
    RMSNormFused,
    VocabParallelEmbedding,
)
from minisgl.layers.base import BaseOP
from minisgl.core import get_global_ctx
from minisgl.utils import nvtx_annotate

from .base import BaseLLMModel
from .config import ModelConfig


def padded_intermediate(inter: int, tp: int) -> int:
    """Intermediate size with each rank's share rounded up to a whole gate/up interleave block.
    The loader fills the extra gate/up rows and down_proj columns with zeros, which contribute
    nothing (act(0) * 0 = 0), so models whose share is not a multiple of the block still load."""
    from minisgl.ops.reference import GATE_UP_BLOCK
    from minisgl.utils import div_even

    local = div_even(inter, tp)
    return -(-local // GATE_UP_BLOCK) * GATE_UP_BLOCK * tp


class GatedMLP(BaseOP):
    def __init__(self, config: ModelConfig, intermediate_size: int | None = None):
        from minisgl.parallel import get_tp_info

        inter = padded_intermediate(intermediate_size or config.intermediate_size, get_tp_info().size)
        self.gate_up_proj = LinearColParallelMerged(config.hidden_size, [inter, inter], has_bias=False)
        if config.hidden_act not in ("silu", "gelu", "gelu_pytorch_tanh"):
            raise ValueError(f"unsupported activation {config.hidden_act}")
        self._act = "silu" if config.hidden_act == "silu" else "gelu"
        self.down_proj = LinearRowParallel(inter, config.hidden_size, has_bias=False)

    @nvtx_annotate("MLP")
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = ops.gate_up_silu(x, self.gate_up_proj.weight, self._act)
        return self.down_proj.forward(y)

    @property
    def output_unreduced(self) -> bool:
        return self.down_proj.deferred


class MoEMLP(BaseOP):
    def __init__(self, config: ModelConfig, router_name: str = "gate", activation: str = "silu",
                 routing: str = "softmax_topk"):
        self.experts = MoELayer(
            num_experts=config.num_experts,
            top_k=config.num_experts_per_tok,
            hidden_size=config.hidden_size,
            intermediate_size=config.moe_intermediate_size,
            renormalize=config.norm_topk_prob,
            activation=activation,
            has_bias=config.mlp_bias,
            routing=routing,
        )
        setattr(self, router_name, LinearReplicated(config.hidden_size, config.num_experts,
                                                    has_bias=config.mlp_bias))
        self._router_name = router_name

    @nvtx_annotate("MoE")
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        router = getattr(self, self._router_name)
        # fp32 router logits: expert choice compares logits that bf16 rounding would tie
        logits = ops.linear_f32(x, router.weight, router.bias)
        return self.experts.forward(x, logits)

    @property
    def output_unreduced(self) -> bool:
        return self.experts.deferred


class RopeAttn(BaseOP):
    def __init__(self, config: ModelConfig, layer_id: int, *, has_attn_bias: bool = False,
                 has_qk_norm: bool = False, has_o_bias: bool = False):
        hd = config.head_dim
        self.qkv_proj = LinearQKVMerged(config.hidden_size, hd, config.num_qo_heads,
                                        config.num_kv_heads, has_bias=has_attn_bias)
        self.q_norm = RMSNorm(hd, config.rms_norm_eps) if has_qk_norm else None
        self.k_norm = RMSNorm(hd, config.rms_norm_eps) if has_qk_norm else None
        self._attn = AttentionLayer(
            layer_id=layer_id, head_dim=hd, num_qo_heads=config.num_qo_heads,
            num_kv_heads=config.num_kv_heads, rotary_config=config.rotary_config,
            q_norm=self.q_norm, k_norm=self.k_norm,
            sliding_window=config.layer_window(layer_id), has_sinks=config.has_sinks,
        )
        if config.has_sinks:
            self.sinks = self._attn.sinks
        self.o_proj = LinearOProj(hd * config.num_qo_heads, config.hidden_size, has_bias=has_o_bias)

    def load_state_dict(self, state_dict, *, prefix: str = "", _internal: bool = False) -> None:
        super().load_state_dict(state_dict, prefix=prefix, _internal=_internal)
        if getattr(self, "sinks", None) is not None:
            self._attn.sinks = self.sinks

    @nvtx_annotate("MHA")
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        qkv = self.qkv_proj.forward(x)
        o = self._attn.forward(qkv)
        return self.o_proj.forward(o)


class DecoderLayer(BaseOP):
    def __init__(self, config: ModelConfig, layer_id: int, *, qk_norm: bool = False,
                 attn_bias: bool = False, o_bias: bool = False, moe: bool = False,
                 moe_kwargs: dict | None = None):
        self.self_attn = RopeAttn(config, layer_id, has_attn_bias=attn_bias, has_qk_norm=qk_norm,
                                  has_o_bias=o_bias)
        self.mlp = MoEMLP(config, **(moe_kwargs or {})) if moe else GatedMLP(config)
        self.input_layernorm = RMSNormFused(config.hidden_size, config.rms_norm_eps)
        self.post_attention_layernorm = RMSNormFused(config.hidden_size, config.rms_norm_eps)
        self._layer_id = layer_id
        # at TP > 1 the row-parallel outputs are reduced by the norms that follow them (fused)
        # (every reduction whose result feeds a norm is deferred to it, so with the NVLS row-sharded
        # form the residual stream is only ever read by the fused norms)
        self.self_attn.o_proj.defer_to_norm = True
        if isinstance(self.mlp, GatedMLP):
            self.mlp.down_proj.defer_to_norm = True
        else:
            self.mlp.experts.defer_to_norm = True

    @nvtx_annotate("Layer_{}", layer_id_field="_layer_id")
    def forward(self, x: torch.Tensor, residual: torch.Tensor | None,
                unreduced: bool = False) -> Tuple[torch.Tensor, torch.Tensor]:
        """``unreduced``: x is the previous layer's partial sum (see LinearRowParallel).
        Returns the MLP output and whether it is still a partial sum."""
        norm = self.input_layernorm
        x, residual = norm.forward_unreduced(x, residual) if unreduced else norm.forward(x, residual)
        x = self.self_attn.forward(x)
        norm = self.post_attention_layernorm
        if self.self_attn.o_proj.deferred:
            x, residual = norm.forward_unreduced(x, residual)
        else:
            x, residual = norm.forward(x, residual)
        x = self.mlp.forward(x)
        return x, residual, self.mlp.output_unreduced


class DecoderModel(BaseOP):
    def __init__(self, config: ModelConfig, **layer_kwargs):
        self.embed_tokens = VocabParallelEmbedding(config.vocab_size, config.hidden_size)
        self.embed_tokens.defer_to_norm = True  # reduced by the first layer's input norm (TP > 1)
        self.layers = OPList([DecoderLayer(config, i, **layer_kwargs) for i in range(config.num_layers)])
        self.norm = RMSNormFused(config.hidden_size, config.rms_norm_eps)

    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        x = self.embed_tokens.forward(input_ids)
        residual = None
        unreduced = self.embed_tokens.deferred
        for layer in self.layers.op_list:
            x, residual, unreduced = layer.forward(x, residual, unreduced)
        if unreduced:
            return self.norm.forward_unreduced(x, residual)[0]
        return self.norm.forward(x, residual)[0]


class DecoderForCausalLM(BaseLLMModel):
    layer_kwargs: dict = {}

    def __init__(self, config: ModelConfig):
        self.model = DecoderModel(config, **self.layer_kwargs)
        tied = self.model.embed_tokens if config.tie_word_embeddings else None
        self.lm_head = ParallelLMHead(config.vocab_size, config.hidden_size,
                                      tie_word_embeddings=config.tie_word_embeddings,
                                      tied_embedding=tied)

    def forward_hidden(self) -> torch.Tensor:
        """The final normalised hidden states (the LM head's input)."""
        return self.model.forward(get_global_ctx().batch.input_ids)

    def forward(self) -> torch.Tensor:
        return self.lm_head.forward(self.forward_hidden())
