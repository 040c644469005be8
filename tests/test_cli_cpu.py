"""Every command-line entry point parses its arguments (``--help`` exits 0) without a GPU."""

import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("cmd", [
    ["-m", "minisgl"],
    ["-m", "minisgl.shell"],
    ["bench.py"],
    ["-m", "minisgl.benchmark.offline"],
    ["-m", "minisgl.benchmark.online"],
    ["-m", "minisgl.benchmark.client"],
    ["-m", "minisgl.benchmark.kernels"],
    ["-m", "minisgl.benchmark.comm"],
    ["-m", "minisgl.models.synthetic"],
])
def test_help(cmd):
    r = subprocess.run([sys.executable] + cmd + ["--help"], cwd=ROOT, env=dict(os.environ, PYTHONPATH=ROOT),
                       capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "usage" in r.stdout.lower()
