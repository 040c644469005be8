import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
os.environ.setdefault("PYTHONPATH", ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "multigpu: needs 2+ GPUs")
    config.addinivalue_line("markers", "slow: long-running")


@pytest.fixture(autouse=True)
def _fresh_globals():
    """Each test starts without a global context / TP identity."""
    from minisgl.core import reset_global_ctx
    from minisgl.parallel.info import reset_tp_info

    reset_global_ctx(None)
    reset_tp_info()
    yield
    reset_global_ctx(None)
    reset_tp_info()
    try:
        import torch.distributed as dist

        if dist.is_initialized():
            dist.destroy_process_group()
    except Exception:
        pass


_PORT = [29600 + (os.getpid() % 200) * 10]


@pytest.fixture
def free_port():
    import socket

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p
