"""Engine configuration (reference: python/minisgl/engine/config.py:15-55).

``device="cpu"`` runs the PyTorch reference ops (oracle / tests); the default runs on
``cuda:<rank>``. ``comm`` selects the TP collective path: ``nccl`` (torch.distributed baseline),
``peer`` (this engine's kernels over CUDA IPC peer memory) or ``auto``.
"""

from __future__ import annotations

from dataclasses import dataclass
from functools import cached_property
from typing import List

import torch

from minisgl.parallel import DistributedInfo


@dataclass(frozen=True)
class EngineConfig:
    model_path: str
    tp_info: DistributedInfo
    dtype: torch.dtype
    max_running_req: int = 256
    attention_backend: str = "auto"
    moe_backend: str = "auto"
    cuda_graph_bs: List[int] | None = None
    cuda_graph_max_bs: int | None = None
    page_size: int = 1
    memory_ratio: float = 0.9
    distributed_timeout: float = 60.0
    use_dummy_weight: bool = False
    use_pynccl: bool = True
    max_seq_len_override: int | None = None
    num_page_override: int | None = None
    device: str | None = None  # None -> cuda:<rank>; "cpu" -> reference ops
    comm: str = "auto"
    dummy_weight_std: float = 0.02
    seed: int = 42
    distributed_port: int = 2333
    external_process_group: bool = False  # torchrun already initialised torch.distributed

    @cached_property
    def hf_config(self):
        from minisgl.utils.hf import cached_load_hf_config

        return cached_load_hf_config(self.model_path)

    @cached_property
    def model_config(self):
        from minisgl.models import ModelConfig

        return ModelConfig.from_hf(self.hf_config)

    @property
    def max_seq_len(self) -> int:
        if self.max_seq_len_override is not None:
            return self.max_seq_len_override
        return self.model_config.rotary_config.max_position

    @property
    def max_forward_len(self) -> int:
        return self.max_seq_len

    @property
    def distributed_addr(self) -> str:
        return f"tcp://127.0.0.1:{self.distributed_port}"
