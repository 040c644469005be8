"""Offline throughput benchmark over the ``LLM`` API: ``python -m minisgl.benchmark.offline``
(reference behaviour: benchmark/offline/bench.py, benchmark/offline/bench_wildchat.py).

Two prompt sources, no downloads:

* ``--dataset FILE``: real conversations, WildChat style. FILE is a parquet shard with a
  ``conversation`` column (a list of turns with ``role`` / ``content`` / ``language`` /
  ``redacted`` / ``toxic``) or JSON lines holding such a ``conversation`` or a plain ``prompt``.
  The first user turn of each conversation is kept if its language is English or Chinese and it
  is neither redacted nor toxic, then rendered with the model's chat template.
* otherwise random token ids with input and output lengths drawn uniformly from ``--input-range``
  and ``--output-range`` (the headline configuration: 256 requests, both U[100, 1024]).

One request runs first as a warm-up; then all requests run in one ``generate`` call, timed on the
host. Prints input / output length statistics and output tokens per second. Under ``torchrun``
every rank runs it (one tensor-parallel group) and rank 0 prints.
"""

from __future__ import annotations

import argparse
import json
import random
import time
from typing import Iterator, List

LANGS = {"English", "Chinese"}


def _first_user_text(conv) -> str | None:
    for turn in conv or []:
        if turn.get("role") != "user":
            continue
        text = (turn.get("content") or "").strip()
        if not text or turn.get("language") not in LANGS:
            return None
        if turn.get("redacted") or turn.get("toxic"):
            return None
        return text
    return None


def iter_dataset_texts(path: str) -> Iterator[str]:
    """First-user-turn prompts of a WildChat-style file (parquet or JSON lines)."""
    if path.endswith(".parquet"):
        import pyarrow.parquet as pq

        f = pq.ParquetFile(path)
        for batch in f.iter_batches(batch_size=256, columns=["conversation"]):
            for conv in batch.to_pydict()["conversation"]:
                text = _first_user_text(conv)
                if text:
                    yield text
        return
    with open(path) as f:
        for line in f:
            if not line.strip():
                continue
            row = json.loads(line)
            text = row.get("prompt") if "prompt" in row else _first_user_text(row.get("conversation"))
            if text:
                yield text


def encode_chat(tokenizer, text: str) -> List[int]:
    """The prompt as the server would tokenize one user message (chat template when the tokenizer
    has one)."""
    from minisgl.tokenizer.tokenize import TokenizeManager

    msg = [{"role": "user", "content": text}] if getattr(tokenizer, "chat_template", None) else text
    return TokenizeManager(tokenizer).encode_one(msg).tolist()


def len_stats(name: str, xs: List[int]) -> str:
    if not xs:
        return f"{name}: no data"
    a = sorted(xs)
    n = len(a)
    return (f"{name}: count={n}, min={a[0]}, p50={a[n // 2]}, p90={a[int(0.9 * n)]}, "
            f"p99={a[min(n - 1, int(0.99 * n))]}, max={a[-1]}")


def _range(s: str):
    lo, hi = (int(x) for x in s.split(","))
    return lo, hi


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser("minisgl.benchmark.offline", description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--model", required=True)
    ap.add_argument("--dataset", default=None)
    ap.add_argument("--num-seqs", type=int, default=256)
    ap.add_argument("--input-range", type=_range, default=(100, 1024))
    ap.add_argument("--output-range", type=_range, default=(100, 1024))
    ap.add_argument("--max-output", type=int, default=4096, help="max_tokens per request with --dataset")
    ap.add_argument("--temperature", type=float, default=None,
                    help="default 0.6 with --dataset (sampled, stops at EOS), greedy otherwise")
    ap.add_argument("--ignore-eos", action="store_true")
    ap.add_argument("--dtype", default="bfloat16")
    ap.add_argument("--device", default="cuda")
    ap.add_argument("--dummy-weight", action="store_true")
    ap.add_argument("--max-running-requests", type=int, default=256)
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)

    import torch

    from minisgl.core import SamplingParams
    from minisgl.llm import LLM
    from minisgl.utils.hf import load_tokenizer

    rng = random.Random(a.seed)
    llm = LLM(a.model, dtype=getattr(torch, a.dtype), device=a.device, use_dummy_weight=a.dummy_weight,
              max_running_req=a.max_running_requests)
    vocab = llm.engine.model_config.vocab_size
    if a.dataset:
        tok = load_tokenizer(a.model)
        prompts = []
        for text in iter_dataset_texts(a.dataset):
            prompts.append(encode_chat(tok, text))
            if len(prompts) >= a.num_seqs:
                break
        temp = 0.6 if a.temperature is None else a.temperature
        sps = [SamplingParams(temperature=temp, ignore_eos=a.ignore_eos, max_tokens=a.max_output, seed=a.seed + i)
               for i in range(len(prompts))]
    else:
        prompts = [[rng.randrange(vocab) for _ in range(rng.randint(*a.input_range))] for _ in range(a.num_seqs)]
        temp = 0.0 if a.temperature is None else a.temperature
        sps = [SamplingParams(temperature=temp, ignore_eos=True, max_tokens=rng.randint(*a.output_range))
               for _ in range(a.num_seqs)]
    try:
        if not prompts:
            raise SystemExit("no prompts (empty dataset after filtering?)")
        llm.generate([prompts[0]], sps[0])  # warm-up
        t = time.perf_counter()
        outs = llm.generate(prompts, sps)
        wall = time.perf_counter() - t
    finally:
        llm.shutdown()
    out_lens = [len(o["token_ids"]) for o in outs]
    res = {"requests": len(prompts), "output_tokens": sum(out_lens), "output_budget": sum(s.max_tokens for s in sps),
           "wall_s": round(wall, 4), "output_tok_per_s": round(sum(out_lens) / wall, 2) if wall > 0 else None}
    if llm.engine.config.tp_info.rank == 0:
        print(len_stats("input length", [len(p) for p in prompts]))
        print(len_stats("output length", out_lens))
        print(json.dumps(res), flush=True)
    return res


if __name__ == "__main__":
    main()
