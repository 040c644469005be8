"""Scheduler configuration (reference: python/minisgl/scheduler/config.py:14-41).

The public fields and their defaults are the reference's: ``max_extend_tokens`` (the prefill chunk
size), ``cache_type`` (``radix`` | ``naive``) and ``offline_mode``. Every ZeroMQ endpoint of one
server is an IPC socket under /tmp named after its channel and the process that built the config,
so two servers on one machine never share a socket and every child process (which receives a copy
of the config) derives the same names.
"""

from __future__ import annotations

import os
from dataclasses import dataclass, field

from minisgl.engine.config import EngineConfig

# channel -> socket number: scheduler input, detokenizer input, rank-0 -> rank-N fan-out,
# frontend input, tokenizer input (the last two are used by the server, minisgl/server/args.py)
IPC_CHANNELS = {"backend": 0, "detokenizer": 1, "broadcast": 2, "frontend": 3, "tokenizer": 4}


@dataclass(frozen=True)
class SchedulerConfig(EngineConfig):
    max_extend_tokens: int = 8192
    cache_type: str = "radix"
    offline_mode: bool = False
    ipc_owner: int = field(default_factory=os.getpid)

    def ipc_addr(self, channel: str) -> str:
        return f"ipc:///tmp/minisgl_{IPC_CHANNELS[channel]}.pid={self.ipc_owner}"

    @property
    def zmq_backend_addr(self) -> str:
        return self.ipc_addr("backend")

    @property
    def zmq_detokenizer_addr(self) -> str:
        return self.ipc_addr("detokenizer")

    @property
    def zmq_scheduler_broadcast_addr(self) -> str:
        return self.ipc_addr("broadcast")

    @property
    def max_forward_len(self) -> int:
        # the longest forward is one full prefill chunk
        return self.max_extend_tokens

    @property
    def scheduler_binds_detokenizer(self) -> bool:
        """Whether rank 0's scheduler creates (binds) the detokenizer socket. Offline and
        single-tokenizer setups have it bind; the server with separate tokenizer workers has the
        detokenizer bind instead."""
        return True
