"""Architecture name -> model class (reference: python/minisgl/models/register.py:5-21)."""

_MODELS = {
    "LlamaForCausalLM": ("minisgl.models.llama", "LlamaForCausalLM"),
    "MistralForCausalLM": ("minisgl.models.llama", "MistralForCausalLM"),
    "Mistral3ForConditionalGeneration": ("minisgl.models.llama", "MistralForCausalLM"),
    "Qwen2ForCausalLM": ("minisgl.models.qwen2", "Qwen2ForCausalLM"),
    "Qwen3ForCausalLM": ("minisgl.models.qwen3", "Qwen3ForCausalLM"),
    "Qwen3MoeForCausalLM": ("minisgl.models.qwen3_moe", "Qwen3MoeForCausalLM"),
    "GptOssForCausalLM": ("minisgl.models.gpt_oss", "GptOssForCausalLM"),
}


def get_model_class(architecture: str):
    import importlib

    if architecture not in _MODELS:
        raise ValueError(f"unsupported architecture {architecture}; supported: {sorted(_MODELS)}")
    mod, cls = _MODELS[architecture]
    return getattr(importlib.import_module(mod), cls)


def supported_architectures():
    return sorted(_MODELS)
