from .config import EngineConfig
from .engine import BatchPlan, Engine, ForwardOutput
from .sample import BatchSamplingArgs, Sampler

__all__ = ["Engine", "EngineConfig", "ForwardOutput", "BatchPlan", "BatchSamplingArgs", "Sampler"]
