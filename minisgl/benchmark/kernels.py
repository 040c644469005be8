"""Kernel micro-benchmarks on one GPU: ``python -m minisgl.benchmark.kernels <op> [options]``.

Each op builds one decode- or prefill-shaped problem, times the kernel with CUDA-graph amplified
events (``perf_cuda``: inputs rotate over buffers larger than L2 where the op streams weights or KV)
and prints one line with time, achieved bandwidth or FLOP/s and the fraction of the measured peaks
in ``MEASURED_PEAKS.json`` (fallback: 6.65 TB/s and 1.59 PFLOP/s). ``--once`` runs the op a few
times without timing, which is the form to wrap in a profiler.

  gemm          bf16 GEMM  out[M, N] = x[M, K] @ w[N, K]^T  (--epi 0 bf16, 1 SiLU-gated, 3 fp32)
  decode-attn   paged decode attention over a longest-first work list (page size 64)
  prefill-attn  ragged causal prefill attention (requests of 100..1024 tokens; --impl tcgen05 | mma)
"""

from __future__ import annotations

import argparse
import json
import math
import os
import random

import torch

from .perf import perf_cuda

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def _peaks() -> tuple[float, float]:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]) * 1e9, float(d["bf16_tflops"]) * 1e12
    except (OSError, KeyError, ValueError):
        return 6.65e12, 1.59e15


def _gemm(a, c) -> None:
    M, N, K, epi = a.m, a.n, a.k, a.epi
    nw = 1 if a.once else max(2, int(3e8 // (N * K * 2)) + 1)
    ws = [torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.02 for _ in range(nw)]
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    nout = N // 2 if epi in (1, 2) else N
    out = torch.empty(M, nout, device="cuda", dtype=torch.float32 if epi == 3 else torch.bfloat16)
    it = [0]

    def run():
        c.gemm(out, x, ws[it[0] % nw], None, epi)
        it[0] += 1

    if a.once:
        for _ in range(4):
            run()
        torch.cuda.synchronize()
        print("ok", c.get_error())
        return
    ms = perf_cuda(run)
    hbm, tf = _peaks()
    flops, nbytes = 2 * M * N * K, (N * K + M * K + M * nout) * 2
    print(f"gemm M={M} N={N} K={K} epi={epi}: {ms * 1e3:.1f} us, {flops / ms / 1e9:.0f} TFLOP/s "
          f"({flops / ms * 1e3 / tf:.2f} of measured), {nbytes / ms / 1e6:.0f} GB/s ({nbytes / ms * 1e3 / hbm:.2f} of measured)")


def _decode_attn(a, c) -> None:
    import numpy as np

    from minisgl.attention.paged import decode_work_list

    random.seed(0)
    bs, nq, nkv, hd, page = a.bs, a.nq, a.nkv, 128, 64
    lens = [random.randint(100, 1500) for _ in range(bs)]
    npages = sum((n + page - 1) // page for n in lens) + 4
    layers = 1 if a.once else max(1, int(6e8 // (npages * page * nkv * hd * 4)) + 1)
    kc = [torch.randn(npages * page, nkv, hd, device="cuda", dtype=torch.bfloat16) for _ in range(layers)]
    vc = [torch.randn(npages * page, nkv, hd, device="cuda", dtype=torch.bfloat16) for _ in range(layers)]
    pt = torch.zeros(bs, (max(lens) + 63) // 64 * 64, dtype=torch.int32)
    perm = torch.randperm(npages)
    k = 0
    for b, n in enumerate(lens):
        for j in range((n + page - 1) // page):
            pt[b, j * page:(j + 1) * page] = perm[k] * page + torch.arange(page)
            k += 1
    pt = pt.cuda()
    rows = torch.arange(bs, dtype=torch.int32, device="cuda")
    kvl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    q = torch.randn(bs, nq, hd, device="cuda", dtype=torch.bfloat16)
    work, n = decode_work_list(np.array(lens), nkv, c.num_sms())
    wd = torch.from_numpy(work).cuda()
    nd = torch.tensor([n], dtype=torch.int32, device="cuda")
    ws = torch.empty(n * nq * (hd + 2), dtype=torch.float32, device="cuda")
    cnt = torch.zeros(bs * nkv, dtype=torch.int32, device="cuda")
    o = torch.empty_like(q)
    it = [0]

    def run():
        i = it[0] % layers
        c.attention_decode_paged(o, q, kc[i], vc[i], pt, rows, kvl, wd, nd, ws, n, cnt, 1 / math.sqrt(hd), -1,
                                 None, page)
        it[0] += 1

    if a.once:
        for _ in range(4):
            run()
        torch.cuda.synchronize()
        print("ok", c.get_error())
        return
    ms = perf_cuda(run)
    hbm, _ = _peaks()
    nbytes = sum(lens) * nkv * hd * 4
    print(f"decode-attn bs={bs} nq={nq} nkv={nkv} avg_len={sum(lens) / bs:.0f}: {ms * 1e3:.1f} us, "
          f"{nbytes / ms / 1e6:.0f} GB/s ({nbytes / ms * 1e3 / hbm:.2f} of measured)")


def _prefill_attn(a, c) -> None:
    random.seed(0)
    nq, nkv, hd, tot = a.nq, a.nkv, 128, a.tokens
    lens = []
    while sum(lens) < tot:
        lens.append(min(random.randint(100, 1024), tot - sum(lens)))
    bs = len(lens)
    kc = torch.randn(tot + 64, nkv, hd, device="cuda", dtype=torch.bfloat16)
    vc = torch.randn(tot + 64, nkv, hd, device="cuda", dtype=torch.bfloat16)
    pt = torch.zeros(bs, 1024, dtype=torch.int32)
    off = 0
    for b, n in enumerate(lens):
        pt[b, :n] = torch.arange(off, off + n)
        off += n
    pt = pt.cuda()
    rows = torch.arange(bs, dtype=torch.int32, device="cuda")
    kvl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    cu = torch.tensor([0] + lens, dtype=torch.int32).cumsum(0).to(torch.int32).cuda()
    q = torch.randn(tot, nq, hd, device="cuda", dtype=torch.bfloat16)
    o = torch.empty_like(q)

    def run():
        if a.impl == "tcgen05":
            c.attention_prefill_fmha(o, q, kc, vc, pt, rows, cu, kvl, max(lens), 1 / math.sqrt(hd), -1, None, 64)
        else:
            c.attention_prefill(o, q, kc, vc, pt, rows, cu, kvl, max(lens), 1 / math.sqrt(hd), -1, None)

    if a.once:
        for _ in range(3):
            run()
        torch.cuda.synchronize()
        print("ok", c.get_error())
        return
    ms = perf_cuda(run, reps=5, graph_calls=3)
    _, tf = _peaks()
    flops = sum(n * (n + 1) / 2 for n in lens) * nq * hd * 4
    print(f"prefill-attn[{a.impl}] tokens={tot} seqs={bs} nq={nq} nkv={nkv}: {ms * 1e3:.1f} us, {flops / ms / 1e9:.0f} TFLOP/s "
          f"({flops / ms * 1e3 / tf:.2f} of measured)")


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("op", choices=["gemm", "decode-attn", "prefill-attn"])
    p.add_argument("--m", type=int, default=128)
    p.add_argument("--n", type=int, default=5120)
    p.add_argument("--k", type=int, default=5120)
    p.add_argument("--epi", type=int, default=0)
    p.add_argument("--bs", type=int, default=128)
    p.add_argument("--nq", type=int, default=40)
    p.add_argument("--nkv", type=int, default=8)
    p.add_argument("--tokens", type=int, default=16384)
    p.add_argument("--impl", default="tcgen05", choices=["tcgen05", "mma"], help="prefill-attn kernel")
    p.add_argument("--once", action="store_true", help="run a few times untimed (for profilers)")
    a = p.parse_args(argv)
    from minisgl._native import cuda

    c = cuda()
    {"gemm": _gemm, "decode-attn": _decode_attn, "prefill-attn": _prefill_attn}[a.op](a, c)


if __name__ == "__main__":
    main()
