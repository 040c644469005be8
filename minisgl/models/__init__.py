from .base import BaseLLMModel
from .config import ModelConfig, RotaryConfig
from .register import get_model_class, supported_architectures


def create_model(config: ModelConfig) -> BaseLLMModel:
    return get_model_class(config.architectures[0])(config)


def load_weight(model_path, device, config=None):
    from .weight import load_weight as _lw

    return _lw(model_path, device, config)


__all__ = [
    "BaseLLMModel",
    "ModelConfig",
    "RotaryConfig",
    "create_model",
    "load_weight",
    "get_model_class",
    "supported_architectures",
]
