"""gpt-oss style MoE decoder (not in the reference): biased attention with learned per-head sinks,
alternating full / sliding-window layers, top-k-then-softmax routing with a biased router, and
experts with biases and the clamped SwiGLU (alpha 1.702, limit 7, ``(up + 1)``)."""

from .utils import DecoderForCausalLM


class GptOssForCausalLM(DecoderForCausalLM):
    layer_kwargs = dict(
        attn_bias=True, o_bias=True, moe=True,
        moe_kwargs=dict(router_name="router", activation="swiglu_oai", routing="topk_softmax"),
    )


__all__ = ["GptOssForCausalLM"]
