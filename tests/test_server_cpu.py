"""The HTTP server end to end on CPU: launcher + tokenizer/detokenizer worker + scheduler process
(reference-op engine) + FastAPI, driven over HTTP like a client would."""

import json
import os
import signal
import subprocess
import sys
import time

import pytest

from minisgl.models.synthetic import make_checkpoint

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _wait_ready(port: int, proc, timeout: float = 120.0) -> None:
    import requests

    t0 = time.time()
    while time.time() - t0 < timeout:
        if proc.poll() is not None:
            raise RuntimeError(proc.stdout.read())
        try:
            if requests.get(f"http://127.0.0.1:{port}/v1/models", timeout=1).status_code == 200:
                return
        except Exception:
            time.sleep(0.5)
    raise TimeoutError("server did not start")


@pytest.mark.parametrize("num_tokenizer", [0, 1])
def test_server_endpoints(tmp_path, free_port, num_tokenizer):
    import requests

    path = make_checkpoint("tiny-qwen3", str(tmp_path / "m"))
    port = free_port
    proc = subprocess.Popen(
        [sys.executable, "-m", "minisgl", "--model", path, "--device", "cpu", "--port", str(port), "--dtype",
         "float32", "--num-tokenizer", str(num_tokenizer), "--max-running-requests", "8"],
        cwd=ROOT, env=dict(os.environ, PYTHONPATH=ROOT), stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
        text=True, start_new_session=True)
    try:
        _wait_ready(port, proc)
        base = f"http://127.0.0.1:{port}"
        assert requests.get(f"{base}/v1").json() == {"status": "ok"}
        assert requests.get(f"{base}/v1/models").json()["data"][0]["id"] == path
        r = requests.post(f"{base}/v1/chat/completions", json={
            "model": "m", "messages": [{"role": "user", "content": "hello"}], "max_tokens": 6,
            "temperature": 0.0, "ignore_eos": True}, timeout=60).json()
        assert r["object"] == "chat.completion" and r["usage"]["completion_tokens"] >= 1
        assert r["usage"]["prompt_tokens"] > 1
        assert r["usage"]["total_tokens"] == r["usage"]["prompt_tokens"] + r["usage"]["completion_tokens"]
        text = r["choices"][0]["message"]["content"]
        # streaming returns the same greedy text in pieces
        chunks = []
        with requests.post(f"{base}/v1/chat/completions", json={
                "model": "m", "messages": [{"role": "user", "content": "hello"}], "max_tokens": 6,
                "temperature": 0.0, "ignore_eos": True, "stream": True}, stream=True, timeout=60) as s:
            for line in s.iter_lines():
                if line.startswith(b"data: ") and line != b"data: [DONE]":
                    chunks.append(json.loads(line[6:]))
        assert chunks[0]["choices"][0]["delta"]["role"] == "assistant"
        assert chunks[-1]["choices"][0]["finish_reason"] == "length"  # ended by max_tokens
        assert "".join(c["choices"][0]["delta"].get("content", "") for c in chunks) == text
        r = requests.post(f"{base}/v1/completions", json={"model": "m", "prompt": "abc", "max_tokens": 4,
                                                          "temperature": 0.0, "ignore_eos": True}, timeout=60).json()
        assert r["object"] == "text_completion"
        with requests.post(f"{base}/generate", json={"prompt": "abc", "max_tokens": 4, "ignore_eos": True},
                           stream=True, timeout=60) as g:
            lines = [l for l in g.iter_lines() if l]
        assert lines[-1] == b"data: [DONE]"
        # a client that disconnects mid-stream aborts its request; the server keeps serving
        with requests.post(f"{base}/generate", json={"prompt": "abc", "max_tokens": 2000, "ignore_eos": True},
                           stream=True, timeout=60) as g:
            next(g.iter_lines())
        time.sleep(0.5)
        r = requests.post(f"{base}/v1/completions", json={"model": "m", "prompt": "x", "max_tokens": 2,
                                                          "temperature": 0.0}, timeout=60)
        assert r.status_code == 200
    finally:
        os.killpg(proc.pid, signal.SIGTERM)
        try:
            proc.wait(timeout=20)
        except subprocess.TimeoutExpired:
            os.killpg(proc.pid, signal.SIGKILL)


def test_trace_readers_and_scaling(tmp_path):
    from minisgl.benchmark.client import read_mooncake_trace, read_qwen_trace, scale_traces
    from minisgl.utils.hf import load_tokenizer

    tok = load_tokenizer(make_checkpoint("tiny-qwen3", str(tmp_path / "m")))
    q = tmp_path / "qwen.jsonl"
    q.write_text("\n".join(json.dumps({"chat_id": i, "parent_chat_id": -1, "timestamp": 100.0 + 0.5 * (3 - i),
                                         "input_length": 5 + 7 * i, "output_length": 3 + i, "type": "text",
                                         "turn": 1, "hash_ids": [i]}) for i in range(4)) + "\n")
    m = tmp_path / "mooncake.jsonl"
    m.write_text("\n".join(json.dumps({"timestamp": 2000 * i, "input_length": 9 + i, "output_length": 4,
                                         "hash_ids": []}) for i in range(3)))
    for shared in (False, True):
        tr = read_qwen_trace(str(q), tok, n=3, shared_text=shared)
        assert [r.input_len for r in tr] == [5, 12, 19] and [r.output_len for r in tr] == [3, 4, 5]
        assert [len(tok.encode(r.prompt, add_special_tokens=False)) for r in tr] == [5, 12, 19]
    sc = scale_traces(tr, 2.0)
    assert [r.arrival for r in sc] == [0.0, 1.0, 2.0] and [r.input_len for r in sc] == [19, 12, 5]
    mc = read_mooncake_trace(str(m), tok)
    assert [r.arrival for r in mc] == [0.0, 2.0, 4.0] and [r.input_len for r in mc] == [9, 10, 11]


def test_bench_client_against_server(tmp_path, free_port, capsys):
    """The online load generator replays a small Poisson trace with shared prefixes and reports
    TTFT / TPOT / E2E percentiles for every request; the CLI's trace-replay and fixed-batch modes
    run against the same server."""
    import asyncio

    from minisgl.benchmark.client import main as client_main
    from minisgl.benchmark.client import run_trace, synthetic_trace
    from minisgl.utils.hf import load_tokenizer

    path = make_checkpoint("tiny-qwen3", str(tmp_path / "m"))
    port = free_port
    proc = subprocess.Popen(
        [sys.executable, "-m", "minisgl", "--model", path, "--device", "cpu", "--port", str(port), "--dtype",
         "float32", "--max-running-requests", "8"],
        cwd=ROOT, env=dict(os.environ, PYTHONPATH=ROOT), stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
        text=True, start_new_session=True)
    try:
        _wait_ready(port, proc)
        tok = load_tokenizer(path)
        trace = synthetic_trace(tok, 12, rate=20.0, in_median=40, in_clip=(16, 120), out_median=6,
                                out_clip=(2, 12), n_prefixes=2, prefix_len=20)
        stats = asyncio.run(run_trace(f"http://127.0.0.1:{port}", trace, path))
        assert stats["completed"] == 12
        assert stats["ttft_p50"] > 0 and stats["tpot_p99"] >= stats["tpot_p50"] >= 0
        tf = tmp_path / "trace.jsonl"
        tf.write_text("\n".join(json.dumps({"timestamp": 0.05 * i, "input_length": 20 + 3 * i, "output_length": 4})
                                 for i in range(6)))
        url = f"http://127.0.0.1:{port}"
        capsys.readouterr()
        client_main(["trace", "--url", url, "--model", path, "--file", str(tf), "--scales", "0.5,1"])
        client_main(["batch", "--url", url, "--model", path, "--batch-size", "5", "--max-input", "60",
                     "--min-output", "2", "--max-output", "6"])
        rows = [json.loads(l) for l in capsys.readouterr().out.splitlines() if l.startswith("{")]
        assert [r.get("scale") for r in rows[:2]] == [0.5, 1.0] and rows[2]["batch_size"] == 5
        assert [r["completed"] for r in rows] == [6, 6, 5]
    finally:
        os.killpg(proc.pid, signal.SIGTERM)
        try:
            proc.wait(timeout=20)
        except subprocess.TimeoutExpired:
            os.killpg(proc.pid, signal.SIGKILL)


def test_server_tp2_matches_tp1(tmp_path, free_port):
    """Two scheduler ranks behind one server (rank 0 receives, publishes the requests to rank 1 and
    broadcasts the message count over gloo every step): the same greedy completions as one rank."""
    import requests

    path = make_checkpoint("tiny-qwen3", str(tmp_path / "m"))
    prompts = ["hello world", "the quick brown fox", "a"]
    texts = {}
    for i, tp in enumerate((1, 2)):
        port = free_port + 20 * i
        proc = subprocess.Popen(
            [sys.executable, "-m", "minisgl", "--model", path, "--device", "cpu", "--port", str(port), "--dtype",
             "float32", "--tp", str(tp), "--max-running-requests", "8"],
            cwd=ROOT, env=dict(os.environ, PYTHONPATH=ROOT), stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
            text=True, start_new_session=True)
        try:
            _wait_ready(port, proc)
            out = []
            for p in prompts:
                r = requests.post(f"http://127.0.0.1:{port}/v1/completions", json={
                    "model": "m", "prompt": p, "max_tokens": 8, "temperature": 0.0, "ignore_eos": True},
                    timeout=60).json()
                out.append(r["choices"][0]["text"])
            texts[tp] = out
        finally:
            os.killpg(proc.pid, signal.SIGTERM)
            try:
                proc.wait(timeout=20)
            except subprocess.TimeoutExpired:
                os.killpg(proc.pid, signal.SIGKILL)
    assert texts[2] == texts[1] and all(texts[1])


def test_stop_strings(tmp_path, free_port):
    """OpenAI ``stop``: the completion ends before the first occurrence of a stop string, in the
    plain and the streamed response alike (the stream holds back text that could still grow into
    a stop string across chunks), and the request is released in the scheduler."""
    import requests

    path = make_checkpoint("tiny-qwen3", str(tmp_path / "m"))
    port = free_port
    proc = subprocess.Popen(
        [sys.executable, "-m", "minisgl", "--model", path, "--device", "cpu", "--port", str(port), "--dtype",
         "float32", "--max-running-requests", "8"],
        cwd=ROOT, env=dict(os.environ, PYTHONPATH=ROOT), stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
        text=True, start_new_session=True)
    try:
        _wait_ready(port, proc)
        url = f"http://127.0.0.1:{port}/v1/completions"
        body = {"model": "m", "prompt": "hello world", "max_tokens": 12, "temperature": 0.0, "ignore_eos": True}
        r0 = requests.post(url, json=body, timeout=60).json()["choices"][0]
        full = r0["text"]
        assert r0["finish_reason"] == "length"  # max_tokens reached (EOS ignored)
        assert len(full) >= 6, full
        stop = full[3:6]
        want = full[: full.find(stop)]
        r1 = requests.post(url, json=dict(body, stop=stop), timeout=60).json()["choices"][0]
        assert r1["text"] == want and r1["finish_reason"] == "stop"
        # max_tokens null means "up to the context limit"; the stop string ends it here
        r2 = requests.post(url, json=dict(body, stop=stop, max_tokens=None), timeout=60).json()["choices"][0]
        assert r2["text"] == want
        pieces = []
        with requests.post(url, json=dict(body, stop=[stop, "\u0000never"], stream=True), stream=True,
                           timeout=60) as s:
            for line in s.iter_lines():
                if line.startswith(b"data: ") and line != b"data: [DONE]":
                    pieces.append(json.loads(line[6:])["choices"][0]["text"])
        assert "".join(pieces) == want
        # stream_options.include_usage: a last chunk with the usage and no choices
        last = None
        with requests.post(url, json=dict(body, stream=True, stream_options={"include_usage": True}), stream=True,
                           timeout=60) as s:
            for line in s.iter_lines():
                if line.startswith(b"data: ") and line != b"data: [DONE]":
                    last = json.loads(line[6:])
        assert last["choices"] == [] and last["usage"]["completion_tokens"] == 12
        assert last["usage"]["prompt_tokens"] > 1
        # the server keeps serving after the early stops
        again = requests.post(url, json=body, timeout=60).json()["choices"][0]["text"]
        assert again == full
        # seeded sampling is reproducible across requests (the noise is keyed by seed, step, token)
        sb = dict(body, temperature=1.0, top_k=50, seed=7)
        a, b = (requests.post(url, json=sb, timeout=60).json()["choices"][0]["text"] for _ in range(2))
        assert a == b
        # n choices: choice i uses seed + i, so choice 0 repeats the single-choice draw
        rn = requests.post(url, json=dict(sb, n=3), timeout=60).json()
        assert [c["index"] for c in rn["choices"]] == [0, 1, 2] and rn["choices"][0]["text"] == a
        assert rn["usage"]["completion_tokens"] == 3 * 12
        one = requests.post(url, json=dict(sb, seed=8), timeout=60).json()["choices"][0]["text"]
        assert rn["choices"][1]["text"] == one
    finally:
        os.killpg(proc.pid, signal.SIGTERM)
        try:
            proc.wait(timeout=20)
        except subprocess.TimeoutExpired:
            os.killpg(proc.pid, signal.SIGKILL)


def test_interactive_shell(tmp_path):
    """``python -m minisgl.shell``: answers each line (the chat history is kept), handles /reset and
    unknown commands, and /exit shuts the backend processes down."""
    path = make_checkpoint("tiny-qwen3", str(tmp_path / "m"))
    env = dict(os.environ, PYTHONPATH=ROOT, MINISGL_SHELL_MAX_TOKENS="4", MINISGL_SHELL_TEMPERATURE="0")
    proc = subprocess.run(
        [sys.executable, "-m", "minisgl.shell", "--model", path, "--device", "cpu", "--dtype", "float32"],
        cwd=ROOT, env=env, input="hello\n/reset\n/foo\nhi again\n/exit\n", capture_output=True, text=True,
        timeout=240)
    out = proc.stdout + proc.stderr
    assert proc.returncode == 0, out[-3000:]
    assert "unknown command /foo" in out and "Exiting shell..." in out, out[-3000:]


def test_online_benchmark_launcher(tmp_path, free_port):
    """``python -m minisgl.benchmark.online`` starts the server, replays Poisson load and reports
    latency statistics per rate, then stops the server."""
    from minisgl.benchmark.online import main

    path = make_checkpoint("tiny-qwen3", str(tmp_path / "m"))
    rows = main(["--model", path, "--port", str(free_port), "--num-requests", "6", "--rates", "20,40",
                 "--in-median", "30", "--out-median", "4", "--prefix-len", "20", "--startup-timeout", "180",
                 "--", "--device", "cpu", "--dtype", "float32", "--max-running-requests", "8"])
    assert [r["rate"] for r in rows] == [20.0, 40.0]
    assert all(r["completed"] == 6 and r["ttft_p50"] > 0 for r in rows)


def test_online_reference_environment():
    """``--impl reference``: the child's ``minisgl`` resolves to the reference installed in
    baseline/_ref, and its API server's prompt_toolkit imports resolve to the stand-in package."""
    import os
    import subprocess
    import sys

    from minisgl.benchmark.online import _reference_env

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    if not os.path.isdir(os.path.join(root, "baseline", "_ref", "minisgl")):
        pytest.skip("reference not installed in baseline/_ref")
    env, cwd = _reference_env()
    code = ("import minisgl, prompt_toolkit; from prompt_toolkit import PromptSession; "
            "from prompt_toolkit.completion import WordCompleter; print(list(minisgl.__path__))")
    out = subprocess.run([sys.executable, "-c", code], env=env, cwd=cwd, capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    assert os.path.join("baseline", "_ref") in out.stdout
