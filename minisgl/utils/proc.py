"""Process lifetime helpers: server processes that end when the process that started them ends.

A killed benchmark launcher (or a killed server main) must not leave a server, its scheduler ranks
or its tokenizer workers running: those hold GPUs and sockets. Linux delivers a chosen signal to a
process when its parent dies (``prctl(PR_SET_PDEATHSIG)``); the server main and every process it
spawns set it, so a kill at the top cascades down the tree.
"""

from __future__ import annotations

import ctypes
import os
import signal
import sys

_PR_SET_PDEATHSIG = 1


def die_with_parent(sig: int = signal.SIGKILL) -> None:
    """Have the kernel send ``sig`` to this process when its parent exits (no-op off Linux). If the
    parent is already gone (this process was re-parented to init) exit at once."""
    if not sys.platform.startswith("linux"):
        return
    parent = os.getppid()
    try:
        libc = ctypes.CDLL(None, use_errno=True)
        libc.prctl(_PR_SET_PDEATHSIG, int(sig), 0, 0, 0)
    except (OSError, AttributeError):
        return
    if parent == 1 or os.getppid() != parent:
        os._exit(1)
