"""Online-serving load generator and latency statistics
(reference behaviour: python/minisgl/benchmark/client.py:18-501, benchmark/online/*.py).

* ``synthetic_trace``: Poisson arrivals at a given rate, lognormal prompt / output lengths with
  clipping, and a fraction of requests that start with one of a few shared prefixes (radix hits).
* ``read_qwen_trace`` / ``read_mooncake_trace``: published serving traces (JSON lines; the Qwen
  Bailian trace gives ``timestamp`` in seconds, Mooncake in milliseconds; both give
  ``input_length`` / ``output_length``), turned into requests with prompts of those lengths.
* ``scale_traces``: rebases a trace to start at 0 and stretches (>1) or compresses (<1) its
  arrival times, which is how one trace is replayed at several loads.
* ``generate_prompt``: text of an exact token length for the engine's tokenizer.
* ``run_trace``: replays a trace against ``/v1/chat/completions`` (or ``/v1/completions``) with
  streaming, records the arrival time of every chunk, and reports TTFT / TPOT / E2E
  (mean, p50, p90, p99, max) and throughput. ``run_batch`` sends a fixed batch at once.

CLI (no downloads: traces are local files)::

    python -m minisgl.benchmark.client synthetic --model M --rates 2,4,8
    python -m minisgl.benchmark.client trace --model M --file qwen_traceA.jsonl --format qwen \
        --scales 0.4,0.5,0.6,0.7,0.8,1.6
    python -m minisgl.benchmark.client batch --model M --batch-size 64 --max-input 8192
"""

from __future__ import annotations

import asyncio
import json
import math
import random
import time
from dataclasses import dataclass, field
from typing import Dict, List, Sequence


@dataclass
class TraceRequest:
    arrival: float  # seconds from start
    prompt: str
    input_len: int
    output_len: int


@dataclass
class RequestResult:
    ok: bool
    start: float
    chunk_times: List[float] = field(default_factory=list)
    output_text: str = ""
    error: str = ""

    @property
    def ttft(self) -> float:
        return self.chunk_times[0] - self.start if self.chunk_times else math.nan

    @property
    def e2e(self) -> float:
        return self.chunk_times[-1] - self.start if self.chunk_times else math.nan

    @property
    def tpots(self) -> List[float]:
        t = self.chunk_times
        return [b - a for a, b in zip(t, t[1:])]


def generate_prompt(tokenizer, n_tokens: int, rng: random.Random) -> str:
    """A text that encodes to ``n_tokens`` tokens (no special tokens): random words, encoded once
    per batch of words (not once per word), cut to ``n_tokens`` ids and decoded."""
    words: List[str] = []
    ids: List[int] = []
    want = max(1, n_tokens)
    while len(ids) < n_tokens:
        words += ["".join(rng.choice("abcdefghijklmnopqrstuvwxyz") for _ in range(rng.randint(2, 8)))
                  for _ in range(want)]
        ids = tokenizer.encode(" ".join(words), add_special_tokens=False)
        want = max(8, n_tokens - len(ids))
    return tokenizer.decode(ids[:n_tokens])


def synthetic_trace(tokenizer, n: int, rate: float, *, in_median: float = 1200, in_sigma: float = 1.0,
                    in_clip=(16, 16384), out_median: float = 250, out_sigma: float = 0.8, out_clip=(1, 2048),
                    shared_frac: float = 0.4, n_prefixes: int = 16, prefix_len: int = 512,
                    seed: int = 0) -> List[TraceRequest]:
    rng = random.Random(seed)
    prefixes = [generate_prompt(tokenizer, prefix_len, rng) for _ in range(n_prefixes)]
    t, out = 0.0, []
    for _ in range(n):
        t += rng.expovariate(rate) if rate > 0 else 0.0
        il = int(min(max(rng.lognormvariate(math.log(in_median), in_sigma), in_clip[0]), in_clip[1]))
        ol = int(min(max(rng.lognormvariate(math.log(out_median), out_sigma), out_clip[0]), out_clip[1]))
        if rng.random() < shared_frac and il > prefix_len + 1:
            body = prefixes[rng.randrange(n_prefixes)] + " " + generate_prompt(tokenizer, il - prefix_len - 1, rng)
        else:
            body = generate_prompt(tokenizer, il, rng)
        out.append(TraceRequest(t, body, il, ol))
    return out


def _prompt_source(tokenizer, lengths: Sequence[int], shared_text: bool, rng: random.Random):
    """Prompt text for each length: fresh random text per request, or (``shared_text``) prefixes
    of one long text, which is quicker to build and gives the radix cache shared prefixes."""
    if not shared_text:
        return [generate_prompt(tokenizer, n, rng) for n in lengths]
    ids = tokenizer.encode(generate_prompt(tokenizer, max(lengths), rng), add_special_tokens=False)
    return [tokenizer.decode(ids[:n]) for n in lengths]


def _read_jsonl(path: str, n: int | None) -> List[dict]:
    rows = []
    with open(path) as f:
        for line in f:
            if line.strip():
                rows.append(json.loads(line))
                if n is not None and len(rows) >= n:
                    break
    return rows


def read_qwen_trace(path: str, tokenizer, n: int | None = None, shared_text: bool = False,
                    seed: int = 0) -> List[TraceRequest]:
    """Qwen Bailian usage trace: one JSON object per line with ``timestamp`` (s), ``input_length``,
    ``output_length`` (its other fields, chat ids, turn, hash ids, are not used)."""
    rows = _read_jsonl(path, n)
    lens = [int(r["input_length"]) for r in rows]
    prompts = _prompt_source(tokenizer, lens, shared_text, random.Random(seed))
    return [TraceRequest(float(r["timestamp"]), p, il, int(r["output_length"]))
            for r, p, il in zip(rows, prompts, lens)]


def read_mooncake_trace(path: str, tokenizer, n: int | None = None, shared_text: bool = False,
                        seed: int = 0) -> List[TraceRequest]:
    """Mooncake trace: ``timestamp`` in milliseconds, ``input_length``, ``output_length``."""
    rows = _read_jsonl(path, n)
    lens = [int(r["input_length"]) for r in rows]
    prompts = _prompt_source(tokenizer, lens, shared_text, random.Random(seed))
    return [TraceRequest(float(r["timestamp"]) / 1000.0, p, il, int(r["output_length"]))
            for r, p, il in zip(rows, prompts, lens)]


def scale_traces(trace: List[TraceRequest], scale: float) -> List[TraceRequest]:
    """Arrival times relative to the first request, multiplied by ``scale``, in arrival order."""
    if not trace:
        return []
    t0 = min(r.arrival for r in trace)
    return sorted((TraceRequest((r.arrival - t0) * scale, r.prompt, r.input_len, r.output_len) for r in trace),
                  key=lambda r: r.arrival)


def _pct(xs: Sequence[float], p: float) -> float:
    xs = sorted(x for x in xs if not math.isnan(x))
    if not xs:
        return math.nan
    k = (len(xs) - 1) * p / 100
    lo, hi = math.floor(k), math.ceil(k)
    return xs[lo] + (xs[hi] - xs[lo]) * (k - lo)


def summarize(results: List[RequestResult], wall: float) -> Dict[str, float]:
    ok = [r for r in results if r.ok and r.chunk_times]
    ttft = [r.ttft for r in ok]
    tpot = [x for r in ok for x in r.tpots]
    e2e = [r.e2e for r in ok]
    out = {"requests": len(results), "completed": len(ok), "wall_s": wall,
           "output_chunks_per_s": sum(len(r.chunk_times) for r in ok) / wall if wall > 0 else math.nan}
    for name, xs in (("ttft", ttft), ("tpot", tpot), ("e2e", e2e)):
        out[f"{name}_mean"] = sum(xs) / len(xs) if xs else math.nan
        for p in (50, 90, 99):
            out[f"{name}_p{p}"] = _pct(xs, p)
        out[f"{name}_max"] = max(xs) if xs else math.nan
    return out


async def _one(session, url: str, req: TraceRequest, model: str, chat: bool, t0: float) -> RequestResult:
    await asyncio.sleep(max(0.0, t0 + req.arrival - time.perf_counter()))
    body = {"model": model, "max_tokens": req.output_len, "temperature": 0.0, "ignore_eos": True, "stream": True}
    if chat:
        body["messages"] = [{"role": "user", "content": req.prompt}]
    else:
        body["prompt"] = req.prompt
    res = RequestResult(ok=False, start=time.perf_counter())
    try:
        async with session.post(url, json=body) as resp:
            async for raw in resp.content:
                line = raw.strip()
                if not line.startswith(b"data: ") or line == b"data: [DONE]":
                    continue
                ch = json.loads(line[6:])["choices"][0]
                piece = ch.get("delta", {}).get("content") if chat else ch.get("text")
                if ch.get("finish_reason") is None:
                    res.chunk_times.append(time.perf_counter())
                    res.output_text += piece or ""
        res.ok = True
    except Exception as e:  # network errors are recorded, not raised
        res.error = repr(e)
    return res


async def run_trace(base_url: str, trace: List[TraceRequest], model: str = "", chat: bool = True) -> Dict[str, float]:
    import aiohttp

    url = base_url.rstrip("/") + ("/v1/chat/completions" if chat else "/v1/completions")
    async with aiohttp.ClientSession(timeout=aiohttp.ClientTimeout(total=None)) as s:
        t0 = time.perf_counter()
        results = await asyncio.gather(*[_one(s, url, r, model, chat, t0) for r in trace])
        wall = time.perf_counter() - t0
    return summarize(list(results), wall)


async def run_batch(base_url: str, prompts: Sequence[str], output_lens: Sequence[int], model: str = "",
                    chat: bool = True) -> Dict[str, float]:
    """All requests at once (a fixed-batch online benchmark)."""
    trace = [TraceRequest(0.0, p, 0, n) for p, n in zip(prompts, output_lens)]
    return await run_trace(base_url, trace, model, chat)


def main(argv=None) -> None:
    import argparse

    from minisgl.utils.hf import load_tokenizer

    ap = argparse.ArgumentParser("minisgl.benchmark.client")
    sub = ap.add_subparsers(dest="mode")
    common = argparse.ArgumentParser(add_help=False)
    common.add_argument("--url", default="http://127.0.0.1:1919")
    common.add_argument("--model", required=True, help="model path (for the tokenizer)")
    common.add_argument("--completions", action="store_true", help="use /v1/completions (no chat template)")
    common.add_argument("--seed", type=int, default=42)
    p = sub.add_parser("synthetic", parents=[common], help="Poisson arrivals at several rates")
    p.add_argument("--num-requests", type=int, default=1000)
    p.add_argument("--rates", default="2,4,8,16,32")
    p = sub.add_parser("trace", parents=[common], help="replay a trace file at several time scales")
    p.add_argument("--file", required=True)
    p.add_argument("--format", choices=["qwen", "mooncake"], default="qwen")
    p.add_argument("--num-requests", type=int, default=1000)
    p.add_argument("--scales", default="0.4,0.5,0.6,0.7,0.8,1.6")
    p = sub.add_parser("batch", parents=[common], help="one fixed batch sent at once")
    p.add_argument("--batch-size", type=int, default=64)
    p.add_argument("--max-input", type=int, default=8192)
    p.add_argument("--min-output", type=int, default=16)
    p.add_argument("--max-output", type=int, default=1024)
    a = ap.parse_args(argv)
    if a.mode is None:
        ap.error("choose a mode: synthetic, trace or batch")
    tok = load_tokenizer(a.model)
    chat = not a.completions

    def emit(tag, stats):
        print(json.dumps({**tag, **{k: round(v, 4) for k, v in stats.items()}}), flush=True)

    if a.mode == "synthetic":
        for rate in [float(x) for x in a.rates.split(",")]:
            trace = synthetic_trace(tok, a.num_requests, rate, seed=a.seed)
            emit({"rate": rate}, asyncio.run(run_trace(a.url, trace, a.model, chat=chat)))
    elif a.mode == "trace":
        reader = read_qwen_trace if a.format == "qwen" else read_mooncake_trace
        base = reader(a.file, tok, n=a.num_requests, shared_text=True, seed=a.seed)
        for scale in [float(x) for x in a.scales.split(",")]:
            emit({"scale": scale}, asyncio.run(run_trace(a.url, scale_traces(base, scale), a.model, chat=chat)))
    else:
        rng = random.Random(a.seed)
        lens = [rng.randint(1, a.max_input) for _ in range(a.batch_size)]
        outs = [rng.randint(a.min_output, a.max_output) for _ in range(a.batch_size)]
        prompts = [generate_prompt(tok, n, rng) for n in lens]
        emit({"batch_size": a.batch_size}, asyncio.run(run_batch(a.url, prompts, outs, a.model, chat=chat)))


if __name__ == "__main__":
    main()
