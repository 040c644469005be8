"""Tensor parallelism: rank identity, collectives, and this engine's peer-memory comm kernels."""

from .comm import DistributedCommunicator, TorchDistributedImpl, destroy_distributed, set_torch_group
from .info import DistributedInfo, get_tp_info, reset_tp_info, set_tp_info, try_get_tp_info

__all__ = [
    "DistributedCommunicator",
    "TorchDistributedImpl",
    "DistributedInfo",
    "destroy_distributed",
    "get_tp_info",
    "reset_tp_info",
    "set_tp_info",
    "set_torch_group",
    "try_get_tp_info",
]
