from .logger import init_logger
from .misc import UNSET, Unset, align_ceil, align_down, call_if_main, div_ceil, div_even
from .registry import Registry
from .torch_utils import nvtx_annotate, torch_dtype

__all__ = [
    "init_logger",
    "Registry",
    "UNSET",
    "Unset",
    "align_ceil",
    "align_down",
    "call_if_main",
    "div_ceil",
    "div_even",
    "nvtx_annotate",
    "torch_dtype",
]


def __getattr__(name):  # lazy: these pull in transformers / zmq
    if name in ("load_tokenizer", "cached_load_hf_config", "download_hf_weight"):
        from . import hf

        return getattr(hf, name)
    if name.startswith("Zmq"):
        from . import mp

        return getattr(mp, name)
    if name in ("is_sm90_supported", "is_sm100_supported"):
        from . import arch

        return getattr(arch, name)
    raise AttributeError(name)
