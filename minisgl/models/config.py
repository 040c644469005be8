"""HF ``PretrainedConfig`` -> frozen ``ModelConfig`` (reference: python/minisgl/models/config.py).

Handles nested ``text_config`` (Mistral3), ``rope_theta`` inside ``rope_scaling``, MoE fields, and
the gpt-oss fields this engine adds (sliding window per layer, attention sinks, biases).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Dict, List, Tuple


@dataclass(frozen=True)
class RotaryConfig:
    head_dim: int
    rotary_dim: int
    max_position: int
    base: float
    scaling: Dict[str, Any] | None


@dataclass(frozen=True)
class ModelConfig:
    num_layers: int
    num_qo_heads: int
    num_kv_heads: int
    head_dim: int
    hidden_size: int
    vocab_size: int
    intermediate_size: int
    rms_norm_eps: float
    rotary_config: RotaryConfig
    hidden_act: str
    tie_word_embeddings: bool
    num_experts: int
    num_experts_per_tok: int
    moe_intermediate_size: int
    norm_topk_prob: bool
    model_type: str
    architectures: List[str]
    attention_bias: bool = False
    sliding_window: int = -1
    layer_types: Tuple[str, ...] = field(default_factory=tuple)
    has_sinks: bool = False
    mlp_bias: bool = False
    quant_method: str | None = None

    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    def layer_window(self, layer_id: int) -> int:
        if self.sliding_window > 0 and self.layer_types:
            return self.sliding_window if self.layer_types[layer_id] == "sliding_attention" else -1
        return -1

    @classmethod
    def from_hf(cls, config) -> "ModelConfig":
        if getattr(config, "text_config", None) is not None:
            top, config = config, config.text_config
            for attr in ("architectures", "rope_theta", "rope_scaling"):
                if not getattr(config, attr, None) and getattr(top, attr, None):
                    setattr(config, attr, getattr(top, attr))
        g = lambda k, d=None: getattr(config, k, d)  # noqa: E731
        heads = config.num_attention_heads
        head_dim = g("head_dim") or config.hidden_size // heads
        rope_scaling = g("rope_scaling") or g("rope_parameters")
        if isinstance(rope_scaling, dict) and rope_scaling.get("rope_type", rope_scaling.get("type")) == "default":
            theta_from = rope_scaling
            rope_scaling = None
        else:
            theta_from = rope_scaling or {}
        rope_theta = g("rope_theta") or theta_from.get("rope_theta", 10000.0)
        model_type = g("model_type", "llama")
        num_experts = g("num_local_experts", g("num_experts", 0)) or 0
        quant = g("quantization_config")
        quant_method = quant.get("quant_method") if isinstance(quant, dict) else None
        layer_types = tuple(g("layer_types") or ())
        return cls(
            num_layers=config.num_hidden_layers,
            num_qo_heads=heads,
            num_kv_heads=g("num_key_value_heads", heads),
            head_dim=head_dim,
            hidden_size=config.hidden_size,
            vocab_size=config.vocab_size,
            intermediate_size=g("intermediate_size", 0) or 0,
            rms_norm_eps=g("rms_norm_eps", 1e-6),
            rotary_config=RotaryConfig(
                head_dim=head_dim,
                rotary_dim=head_dim,
                max_position=g("max_position_embeddings", 4096),
                base=float(rope_theta),
                scaling=dict(rope_scaling) if rope_scaling else None,
            ),
            hidden_act=g("hidden_act", "silu"),
            tie_word_embeddings=bool(g("tie_word_embeddings", False)),
            num_experts=num_experts,
            num_experts_per_tok=g("num_experts_per_tok", g("experts_per_token", 0)) or 0,
            moe_intermediate_size=g("moe_intermediate_size", 0) or (g("intermediate_size", 0) if model_type == "gpt_oss" else 0),
            norm_topk_prob=bool(g("norm_topk_prob", False)),
            model_type=model_type,
            architectures=list(g("architectures") or ["LlamaForCausalLM"]),
            attention_bias=bool(g("attention_bias", False)) or model_type == "qwen2",
            sliding_window=int(g("sliding_window") or -1) if layer_types else -1,
            layer_types=layer_types,
            has_sinks=model_type == "gpt_oss",
            mlp_bias=model_type == "gpt_oss",
            quant_method=quant_method,
        )
