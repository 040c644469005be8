"""Command-line flags -> ``ServerArgs`` (reference: python/minisgl/server/args.py:14-268).

Same flag names as the reference, plus ``--device`` (``cpu`` runs the reference-op engine),
``--comm`` (``auto`` | ``nccl`` | ``peer``) and ``--distributed-timeout``.
"""

from __future__ import annotations

import argparse
from dataclasses import dataclass, fields
from typing import List

import torch

from minisgl.parallel import DistributedInfo
from minisgl.scheduler.config import SchedulerConfig


@dataclass(frozen=True)
class ServerArgs(SchedulerConfig):
    server_host: str = "127.0.0.1"
    server_port: int = 1919
    num_tokenizer: int = 0
    silent_output: bool = False
    shell_mode: bool = False
    model_source: str = "huggingface"

    @property
    def share_tokenizer(self) -> bool:
        return self.num_tokenizer == 0

    @property
    def zmq_frontend_addr(self) -> str:
        return self.ipc_addr("frontend")

    @property
    def zmq_tokenizer_addr(self) -> str:
        return self.zmq_detokenizer_addr if self.share_tokenizer else self.ipc_addr("tokenizer")

    @property
    def tokenizer_create_addr(self) -> bool:
        return self.share_tokenizer

    @property
    def scheduler_binds_detokenizer(self) -> bool:
        return not self.share_tokenizer

    @property
    def frontend_create_tokenizer_link(self) -> bool:
        return not self.share_tokenizer


_DTYPES = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}


def _resolve_dtype(name: str, model_path: str) -> torch.dtype:
    if name != "auto":
        return _DTYPES[name]
    try:
        from minisgl.utils.hf import cached_load_hf_config

        cfg = cached_load_hf_config(model_path)
        d = getattr(cfg, "torch_dtype", None) or getattr(cfg, "dtype", None)
        d = str(d).replace("torch.", "") if d is not None else "bfloat16"
    except Exception:
        d = "bfloat16"
    return torch.float16 if d in ("float32", "float16") else torch.bfloat16


def build_parser() -> argparse.ArgumentParser:
    from minisgl.attention import SUPPORTED_ATTENTION_BACKENDS
    from minisgl.kvcache import SUPPORTED_CACHE_MANAGER
    from minisgl.moe import SUPPORTED_MOE_BACKENDS

    d = ServerArgs
    p = argparse.ArgumentParser("minisgl", description="B200-native mini-sglang server")
    p.add_argument("--model-path", "--model", dest="model_path", required=True)
    p.add_argument("--dtype", default="auto", choices=["auto", "float16", "bfloat16", "float32"])
    p.add_argument("--tensor-parallel-size", "--tp-size", "--tp", dest="tp_size", type=int, default=1)
    p.add_argument("--max-running-requests", dest="max_running_req", type=int, default=d.max_running_req)
    p.add_argument("--max-seq-len-override", type=int, default=d.max_seq_len_override)
    p.add_argument("--memory-ratio", type=float, default=d.memory_ratio)
    p.add_argument("--dummy-weight", dest="use_dummy_weight", action="store_true")
    p.add_argument("--disable-pynccl", dest="use_pynccl", action="store_false")
    p.add_argument("--host", dest="server_host", default=d.server_host)
    p.add_argument("--port", dest="server_port", type=int, default=d.server_port)
    p.add_argument("--cuda-graph-max-bs", "--graph", dest="cuda_graph_max_bs", type=int, default=d.cuda_graph_max_bs)
    p.add_argument("--num-tokenizer", "--tokenizer-count", dest="num_tokenizer", type=int, default=d.num_tokenizer)
    p.add_argument("--max-prefill-length", "--max-extend-length", dest="max_extend_tokens", type=int,
                   default=d.max_extend_tokens)
    p.add_argument("--num-pages", dest="num_page_override", type=int, default=d.num_page_override)
    p.add_argument("--page-size", type=int, default=d.page_size)
    p.add_argument("--attention-backend", "--attn", dest="attention_backend", default=d.attention_backend,
                   help=f"accepted for compatibility: {SUPPORTED_ATTENTION_BACKENDS.supported_names()} "
                        "(all run this engine's kernels)")
    p.add_argument("--model-source", default="huggingface", choices=["huggingface", "modelscope"])
    p.add_argument("--cache-type", default=d.cache_type, choices=SUPPORTED_CACHE_MANAGER.supported_names())
    p.add_argument("--moe-backend", default=d.moe_backend, choices=SUPPORTED_MOE_BACKENDS.supported_names())
    p.add_argument("--shell-mode", action="store_true")
    p.add_argument("--device", default=None, help="cuda (default) or cpu (reference ops, for testing)")
    p.add_argument("--comm", default=d.comm, choices=["auto", "nccl", "peer", "fused"])
    p.add_argument("--distributed-timeout", type=float, default=d.distributed_timeout)
    p.add_argument("--silent-output", action="store_true")
    return p


def parse_args(argv: List[str], run_shell: bool = False) -> ServerArgs:
    a = build_parser().parse_args(argv)
    from minisgl.attention import validate_attn_backend

    validate_attn_backend(a.attention_backend)
    if a.model_source == "modelscope":
        try:
            from modelscope import snapshot_download  # noqa: F401
        except ImportError:
            raise SystemExit("--model-source modelscope needs the modelscope package")
    kw = {f.name: getattr(a, f.name) for f in fields(ServerArgs) if f.init and hasattr(a, f.name)}
    kw.pop("tp_info", None)
    kw["dtype"] = _resolve_dtype(a.dtype, a.model_path)
    kw["tp_info"] = DistributedInfo(0, a.tp_size)
    kw["distributed_port"] = a.server_port + 1
    kw["shell_mode"] = a.shell_mode or run_shell
    if kw["shell_mode"]:  # one interactive request at a time
        kw["cuda_graph_max_bs"] = 1
        kw["max_running_req"] = 1
    return ServerArgs(**kw)
