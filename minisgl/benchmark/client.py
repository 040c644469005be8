"""Online-serving load generator and latency statistics
(reference behaviour: python/minisgl/benchmark/client.py:18-501).

* ``synthetic_trace``: Poisson arrivals at a given rate, lognormal prompt / output lengths with
  clipping, and a fraction of requests that start with one of a few shared prefixes (radix hits).
* ``generate_prompt``: text of an exact token length for the engine's tokenizer.
* ``run_trace``: replays a trace against ``/v1/chat/completions`` (or ``/v1/completions``) with
  streaming, records the arrival time of every chunk, and reports TTFT / TPOT / E2E
  (mean, p50, p90, p99, max) and throughput.
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
    """A text that encodes to ``n_tokens`` tokens (no special tokens)."""
    words: List[str] = []
    while True:
        words.append("".join(rng.choice("abcdefghijklmnopqrstuvwxyz") for _ in range(rng.randint(2, 8))))
        if len(tokenizer.encode(" ".join(words), add_special_tokens=False)) >= n_tokens:
            break
    ids = tokenizer.encode(" ".join(words), add_special_tokens=False)[:n_tokens]
    return tokenizer.decode(ids)


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


def main() -> None:
    import argparse

    from minisgl.utils.hf import load_tokenizer

    ap = argparse.ArgumentParser("minisgl.benchmark.client")
    ap.add_argument("--url", default="http://127.0.0.1:1919")
    ap.add_argument("--model", required=True, help="model path (for the tokenizer)")
    ap.add_argument("--num-requests", type=int, default=1000)
    ap.add_argument("--rates", default="2,4,8,16,32")
    ap.add_argument("--completions", action="store_true", help="use /v1/completions (no chat template)")
    a = ap.parse_args()
    tok = load_tokenizer(a.model)
    for rate in [float(x) for x in a.rates.split(",")]:
        trace = synthetic_trace(tok, a.num_requests, rate)
        stats = asyncio.run(run_trace(a.url, trace, a.model, chat=not a.completions))
        print(json.dumps({"rate": rate, **{k: round(v, 4) for k, v in stats.items()}}), flush=True)


if __name__ == "__main__":
    main()
