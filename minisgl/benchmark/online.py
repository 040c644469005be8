"""Online serving benchmark in one command: start the server, replay load, report latencies.

    python -m minisgl.benchmark.online --model M [--tp 4] [--rates 2,4,8 | --trace FILE --scales ...]
        [-- extra server flags]

Launches ``python -m minisgl`` (this engine, or with ``--impl reference`` the unmodified reference
from baseline/_ref) as a child process group (its own session, stopped at the end),
waits until ``/v1/models`` answers, then drives it with the client of ``minisgl.benchmark.client``:
Poisson arrivals at each rate with lognormal prompt / output lengths and shared prefixes, or a
Qwen-Bailian / Mooncake trace file replayed at each time scale. Prints one JSON line per load
point with TTFT / TPOT / E2E statistics (the reference's online scripts, benchmark/online/*.py,
expect an already running server and download the trace; this one uses local files only).
"""

from __future__ import annotations

import argparse
import asyncio
import json
import os
import signal
import subprocess
import sys
import time
import urllib.request


def wait_ready(port: int, proc: subprocess.Popen, timeout: float) -> None:
    t0 = time.time()
    while time.time() - t0 < timeout:
        if proc.poll() is not None:
            raise RuntimeError(f"server exited with code {proc.returncode}")
        try:
            with urllib.request.urlopen(f"http://127.0.0.1:{port}/v1/models", timeout=1) as r:
                if r.status == 200:
                    return
        except OSError:
            time.sleep(0.5)
    raise TimeoutError(f"server not ready after {timeout:.0f} s")


def _reference_env():
    """Environment that makes ``python -m minisgl`` resolve to the reference installed in
    baseline/_ref. Its API server imports prompt_toolkit at load time for the interactive shell,
    which this image lacks; a stand-in package that only defines the two imported names (and fails
    if the shell is used) lets the HTTP server start. The reference's code is not modified."""
    import tempfile

    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    ref = os.path.join(root, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "minisgl")):
        raise SystemExit("the reference is not installed in baseline/_ref")
    stub = tempfile.mkdtemp(prefix="minisgl_ref_stub_")
    os.makedirs(os.path.join(stub, "prompt_toolkit"))
    with open(os.path.join(stub, "prompt_toolkit", "__init__.py"), "w") as f:
        f.write("class PromptSession:\n    def __init__(self, *a, **k):\n"
                "        raise RuntimeError('interactive shell unavailable: prompt_toolkit is not installed')\n")
    with open(os.path.join(stub, "prompt_toolkit", "completion.py"), "w") as f:
        f.write("class WordCompleter:\n    def __init__(self, *a, **k):\n        pass\n")
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([ref, stub])
    return env, stub  # run from outside this repository so its package does not shadow the reference


def main(argv=None) -> list:
    argv = list(sys.argv[1:] if argv is None else argv)
    extra = []
    if "--" in argv:
        i = argv.index("--")
        argv, extra = argv[:i], argv[i + 1:]
    ap = argparse.ArgumentParser("minisgl.benchmark.online", description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--model", required=True)
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--port", type=int, default=1919)
    ap.add_argument("--num-requests", type=int, default=1000)
    ap.add_argument("--rates", default="2,4,8,16,32", help="Poisson arrival rates (req/s)")
    ap.add_argument("--trace", default=None, help="trace file (JSON lines) instead of Poisson arrivals")
    ap.add_argument("--format", choices=["qwen", "mooncake"], default="qwen")
    ap.add_argument("--scales", default="0.4,0.5,0.6,0.7,0.8,1.6")
    ap.add_argument("--in-median", type=float, default=1200)
    ap.add_argument("--out-median", type=float, default=250)
    ap.add_argument("--prefix-len", type=int, default=512, help="length of the shared prompt prefixes")
    ap.add_argument("--startup-timeout", type=float, default=1800)
    ap.add_argument("--seed", type=int, default=42)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours",
                    help="serve with this engine, or with the unmodified reference installed in baseline/_ref")
    a = ap.parse_args(argv)

    from minisgl.benchmark.client import (read_mooncake_trace, read_qwen_trace, run_trace, scale_traces,
                                          synthetic_trace)
    from minisgl.utils.hf import load_tokenizer

    cmd = [sys.executable, "-m", "minisgl", "--model", a.model, "--tp", str(a.tp), "--port", str(a.port)] + extra
    env, cwd = None, None
    if a.impl == "reference":
        env, cwd = _reference_env()
    from minisgl.utils.proc import die_with_parent

    # its own process group (killed as a group below), and killed by the kernel if this launcher dies
    # first (a timeout or a signal skips the finally clause)
    proc = subprocess.Popen(cmd, start_new_session=True, preexec_fn=die_with_parent, env=env, cwd=cwd)
    rows = []
    try:
        wait_ready(a.port, proc, a.startup_timeout)
        tok = load_tokenizer(a.model)
        url = f"http://127.0.0.1:{a.port}"
        if a.trace:
            reader = read_qwen_trace if a.format == "qwen" else read_mooncake_trace
            base = reader(a.trace, tok, n=a.num_requests, shared_text=True, seed=a.seed)
            points = [({"scale": float(x)}, scale_traces(base, float(x))) for x in a.scales.split(",")]
        else:
            points = [({"rate": float(x)}, synthetic_trace(tok, a.num_requests, float(x), in_median=a.in_median,
                                                            out_median=a.out_median, prefix_len=a.prefix_len,
                                                            seed=a.seed))
                      for x in a.rates.split(",")]
        for tag, trace in points:
            stats = asyncio.run(run_trace(url, trace, a.model))
            row = {"tp": a.tp, **tag, **{k: round(v, 4) for k, v in stats.items()}}
            rows.append(row)
            print(json.dumps(row), flush=True)
    finally:
        try:
            os.killpg(proc.pid, signal.SIGTERM)
            proc.wait(timeout=30)
        except (ProcessLookupError, subprocess.TimeoutExpired):
            try:
                os.killpg(proc.pid, signal.SIGKILL)
            except ProcessLookupError:
                pass
    return rows


if __name__ == "__main__":
    main()
