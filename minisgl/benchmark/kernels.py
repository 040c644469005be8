"""Kernel micro-benchmarks on one GPU: ``python -m minisgl.benchmark.kernels <op> [options]``.

Each op builds one decode- or prefill-shaped problem, times the kernel with CUDA-graph amplified
events (``perf_cuda``: inputs rotate over buffers larger than L2 where the op streams weights or KV)
and prints one line with time, achieved bandwidth or FLOP/s and the fraction of the measured peaks
in ``MEASURED_PEAKS.json`` (fallback: 6.65 TB/s and 1.59 PFLOP/s). ``--once`` runs the op a few
times without timing, which is the form to wrap in a profiler.

  gemm          bf16 GEMM  out[M, N] = x[M, K] @ w[N, K]^T  (--epi 0 bf16, 1 SiLU-gated, 3 fp32)
  gemm-sweep    Qwen3-14B decode GEMMs per TP degree: automatic plan vs every forced tiling vs cuBLAS
  decode-attn   paged decode attention over a longest-first work list (page size 64)
  prefill-attn  ragged causal prefill attention (requests of 100..1024 tokens; --impl tcgen05 | mma | trtllm)
  moe           one gpt-oss-style MoE layer, experts bf16 vs MXFP4 kept in fp4
  suite         every other hot kernel once at decode shapes (Qwen3-14B, --bs tokens; MoE at
                Qwen3-30B-A3B shapes): embedding, RMSNorm, fused add+RMSNorm, QK-norm+RoPE+KV
                store, KV store, SiLU-mul, 1-SM and 2-SM GEMMs, argmax, top-k/top-p sampling and
                the MoE route / align / gather / grouped GEMM / activation / combine chain
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
    if a.impl == "trtllm":  # FlashInfer's trtllm-gen context kernel on the same requests (64-token pages)
        from flashinfer.prefill import trtllm_batch_context_with_kv_cache

        npg = [(n + 63) // 64 for n in lens]
        kp = torch.randn(sum(npg), 64, nkv, hd, device="cuda", dtype=torch.bfloat16)
        vp = torch.randn_like(kp)
        bt = torch.zeros(bs, max(npg), dtype=torch.int32)
        first = 0
        for b_, m_ in enumerate(npg):
            bt[b_, :m_] = torch.arange(first, first + m_)
            first += m_
        bt = bt.cuda()
        fi_ws = torch.empty(128 << 20, dtype=torch.uint8, device="cuda")

    def run():
        if a.impl == "trtllm":
            trtllm_batch_context_with_kv_cache(
                query=q, kv_cache=(kp, vp), workspace_buffer=fi_ws, block_tables=bt, seq_lens=kvl,
                max_q_len=max(lens), max_kv_len=max(lens), bmm1_scale=1 / math.sqrt(hd), bmm2_scale=1.0,
                cum_seq_lens_q=cu, cum_seq_lens_kv=cu, kv_layout="NHD", batch_size=bs, out_dtype=q.dtype)
        elif a.impl == "tcgen05":
            c.attention_prefill_fmha(o, q, kc, vc, pt, rows, cu, kvl, max(lens), 1 / math.sqrt(hd), -1, None, 64)
        else:
            c.attention_prefill(o, q, kc, vc, pt, rows, cu, kvl, max(lens), 1 / math.sqrt(hd), -1, None)

    if a.once:
        for _ in range(3):
            run()
        torch.cuda.synchronize()
        print("ok", c.get_error())
        return
    if a.trace and a.impl == "tcgen05":
        _prefill_trace(c, run, a.trace_file)
        return
    ms = perf_cuda(run, reps=5, graph_calls=3)
    _, tf = _peaks()
    flops = sum(n * (n + 1) / 2 for n in lens) * nq * hd * 4
    print(f"prefill-attn[{a.impl}] tokens={tot} seqs={bs} nq={nq} nkv={nkv}: {ms * 1e3:.1f} us, {flops / ms / 1e9:.0f} TFLOP/s "
          f"({flops / ms * 1e3 / tf:.2f} of measured)")


def _prefill_trace(c, run, path=None) -> None:
    """Median phase durations (SM cycles) of one tile (the third) of each persistent CTA of the
    tcgen05 prefill kernel, from its clock stamps (slot map beside ``kFmTrace`` in ``attention.cu``),
    and the spread of the CTAs' total times (load balance)."""
    import statistics

    run()  # warm
    torch.cuda.synchronize()
    tr = torch.zeros(2048, 96, dtype=torch.int32, device="cuda")
    c.attention_prefill_trace(tr)
    run()
    torch.cuda.synchronize()
    c.attention_prefill_trace(None)
    import numpy as np

    t = tr.cpu().numpy().astype("int64")
    t = t[t[:, 82] > 0]
    if path:
        np.save(path, t)
    rows = []

    def med(name, vals):
        vals = [int(v) for v in vals]
        if vals:
            rows.append((name, statistics.median(vals), len(vals)))

    med("traced tile published", t[:, 1])
    med("softmax idle at the tile start", t[:, 40] - t[:, 88])
    med("MMA took the tile, after publish", t[:, 89] - t[:, 1])
    for k, name in ((90, "Q"), (91, "K0"), (92, "S buffer free"), (93, "PV within 2")):
        med(f"first S input ready: {name}, after MMA took the tile", t[:, k] - t[:, 89])
    med("first S issued, after MMA took the tile", t[:, 24] - t[:, 89])
    med("Q issued after publish", t[:, 3] - t[:, 1])
    med("K0 issued after publish", t[:, 8] - t[:, 1])
    med("S0 issued after K0 issue", t[:, 24] - t[:, 8])
    med("S0 landed in softmax after issue", t[:, 40] - t[:, 24])
    for i in range(6):
        sel = t[t[:, 2] > i]
        if len(sel) == 0:
            break
        s0 = 40 + 4 * i
        med(f"blk{i}: softmax idle before S", (sel[:, s0] - sel[:, s0 - 1]) if i else sel[:, s0] - sel[:, 1])
        med(f"blk{i}: S load + max", sel[:, s0 + 1] - sel[:, s0])
        med(f"blk{i}: exp + sum", sel[:, s0 + 2] - sel[:, s0 + 1])
        med(f"blk{i}: P store + hand-over", sel[:, s0 + 3] - sel[:, s0 + 2])
        med(f"blk{i}: S issued after K issued", sel[:, 24 + i] - sel[:, 8 + i])
        med(f"blk{i}: PV issued after P handed", sel[:, 32 + i] - sel[:, s0 + 3])
        med(f"blk{i}: V issued after K issued", sel[:, 16 + i] - sel[:, 8 + i])
    last = [int(r[40 + 4 * (int(r[2]) - 1) + 3]) if 0 < r[2] <= 8 else None for r in t]
    med("last PV done after last P", [r[80] - l for r, l in zip(t, last) if l is not None])
    med("O stored", t[:, 81] - t[:, 80])
    med("CTA total (all its tiles)", t[:, 82])
    med("key blocks of the traced tile", t[:, 2])
    for name, v, n in rows:
        print(f"{name:40s} {v:10.0f}  (n={n})")
    sms = {}
    for r in t:
        sms.setdefault(int(r[6]), []).append((int(r[7]), int(r[83])))
    conc = []
    for iv in sms.values():  # most CTAs resident on one SM at once
        ev = sorted([(a, 1) for a, _ in iv] + [(b, -1) for _, b in iv])
        cur = best = 0
        for _, d in ev:
            cur += d
            best = max(best, cur)
        conc.append(best)
    tiles = sorted(int(v) for v in t[:, 84])
    span = (max(int(v) for v in t[:, 83]) - min(int(v) for v in t[:, 7])) * 32 / 1e3
    print(f"SMs used {len(sms)}, CTAs resident per SM (max) {max(conc)}, (min) {min(conc)}; tiles per CTA "
          f"min / median / max {tiles[0]} / {tiles[len(tiles) // 2]} / {tiles[-1]} (sum {sum(tiles)}); "
          f"first start to last end {span:.1f} us")
    stuck = t[t[:, 84] == 0]
    if len(stuck):
        print(f"CTAs without a tile: {len(stuck)}; their median cycles to TMEM alloc / past the launch wait / "
              f"first fetch: {np.median(stuck[:, 85]):.0f} / {np.median(stuck[:, 86]):.0f} / {np.median(stuck[:, 87]):.0f}")
    tot = sorted(int(v) for v in t[:, 82])
    print(f"CTA totals min / median / max: {tot[0]} / {tot[len(tot) // 2]} / {tot[-1]}; "
          f"dynamic smem base mod 1024: {sorted(set(int(v) for v in t[:, 5]))}")


def _moe(a, c) -> None:
    """One gpt-oss-style MoE layer (swiglu_oai, biases, top-k after softmax) on ``--bs`` tokens:
    experts as bf16 vs MXFP4 kept in fp4 (converted inside the grouped GEMM). Reports CUDA-event
    time per layer and the expert bytes read per call (experts hit by the routing, all of their
    rows) as a fraction of the measured HBM bandwidth."""
    from minisgl.moe.mxfp4 import Mxfp4Experts, interleave_rows, pad_k
    from minisgl.ops.moe import interleave_experts, moe_forward

    E, H, inter, T, topk = a.experts, a.hidden, a.inter, a.bs, a.topk
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(0)
    b1 = torch.randint(0, 256, (E, 2 * inter, H // 32, 16), generator=g, device=dev, dtype=torch.uint8)
    s1 = torch.randint(119, 124, (E, 2 * inter, H // 32), generator=g, device=dev, dtype=torch.uint8)
    b2 = torch.randint(0, 256, (E, H, inter // 32, 16), generator=g, device=dev, dtype=torch.uint8)
    s2 = torch.randint(119, 124, (E, H, inter // 32), generator=g, device=dev, dtype=torch.uint8)
    q1 = Mxfp4Experts.pack(interleave_rows(b1), interleave_rows(s1), 256)
    ip = q1.n // 2
    q2 = Mxfp4Experts.pack(*pad_k(b2, s2, ip), 128)
    del b1, s1, b2, s2
    x = torch.randn(T, H, device=dev, dtype=torch.bfloat16)
    gating = torch.randn(T, E, device=dev)
    bias1 = torch.zeros(E, 2 * ip, device=dev, dtype=torch.bfloat16)
    bias2 = torch.zeros(E, H, device=dev, dtype=torch.bfloat16)
    hit = int(torch.topk(gating, topk, dim=-1).indices.unique().numel())
    hbm, _ = _peaks()
    impls = {"mxfp4": (q1, q2)}
    if not a.once:
        w1 = q1.dequant()
        w2 = q2.dequant()
        impls["bf16"] = (w1, w2)
    for name, (w1, w2) in impls.items():
        def run():
            moe_forward(x, w1, w2, gating, topk, True, "swiglu_oai", bias1, bias2, True, 0, True)

        if a.once:
            for _ in range(3):
                run()
            torch.cuda.synchronize()
            print("ok", c.get_error())
            return
        ms = perf_cuda(run, reps=10, graph_calls=5)
        per_expert = (q1.nbytes() + q2.nbytes()) / E if name == "mxfp4" else (w1.numel() + w2.numel()) * 2 / E
        nbytes = per_expert * hit
        print(f"moe[{name}] tokens={T} experts={E} hit={hit} H={H} I={inter} top{topk}: {ms * 1e3:.1f} us, "
              f"{nbytes / ms / 1e6:.0f} GB/s of expert weights ({nbytes / ms * 1e3 / hbm:.2f} of measured)")


def _suite(a, c) -> None:
    """One table row per kernel: CUDA-event time (graph replay) and bytes the kernel must move.
    Weight-streaming entries rotate over copies larger than L2; activation-sized entries are
    latency-bound and run L2-resident, as they do inside a decode step."""
    from minisgl import ops
    from minisgl.layers.rotary import get_rope

    torch.manual_seed(0)
    dev, bf = "cuda", torch.bfloat16
    T, H, nq, nkv, hd, inter, V = a.bs, 5120, 40, 8, 128, 17408, 151936
    small = a.once  # smaller weights under a profiler (few GB on the device)
    rows = []

    def add(name, fn, nbytes):
        if a.once:
            fn()
            return
        ms = perf_cuda(fn)
        rows.append((name, ms * 1e3, nbytes / ms / 1e6))

    def rot(make, n):
        bufs = [make() for _ in range(n)]
        it = [0]

        def nxt():
            it[0] += 1
            return bufs[it[0] % n]
        return nxt

    nrot = lambda nb: 1 if small else max(2, int(3e8 // nb) + 1)  # noqa: E731
    # embedding (vocab gather)
    Vs = 32000 if small else V
    emb = torch.randn(Vs, H, device=dev, dtype=bf)
    ids = torch.randint(0, Vs, (T,), device=dev, dtype=torch.int32)
    add("embedding", lambda: ops.embedding(emb, ids), 2 * T * H * 2)
    x = torch.randn(T, H, device=dev, dtype=bf)
    w = torch.rand(H, device=dev, dtype=bf) + 0.5
    res = torch.randn(T, H, device=dev, dtype=bf)
    add("rmsnorm", lambda: ops.rmsnorm(x, w, 1e-6), 2 * T * H * 2)
    add("fused_add_rmsnorm", lambda: ops.fused_add_rmsnorm(x, res, w, 1e-6), 4 * T * H * 2)
    # attention input: QK-norm + RoPE + KV store, and the plain KV store
    slots = 65536
    kc = torch.zeros(slots, nkv, hd, device=dev, dtype=bf)
    vc = torch.zeros_like(kc)
    qkv = torch.randn(T, (nq + 2 * nkv) * hd, device=dev, dtype=bf)
    pos = torch.randint(0, 4000, (T,), device=dev, dtype=torch.int32)
    loc = torch.randperm(slots, device=dev)[:T].to(torch.int32)
    cs = get_rope(hd, hd, 4096, 1e6).cos_sin_cache.to(dev)
    qn = torch.rand(hd, device=dev, dtype=bf) + 0.5
    add("qk_norm_rope_store", lambda: ops.qk_norm_rope_store(qkv, pos, cs, qn, qn, 1e-6, kc, vc, loc, nq, nkv, hd),
        2 * qkv.numel() * 2)
    k = torch.randn(T, nkv * hd, device=dev, dtype=bf)
    add("store_kv", lambda: ops.store_kv(k, k, kc, vc, loc), 4 * k.numel() * 2)
    gu = torch.randn(T, 2 * inter, device=dev, dtype=bf)
    add("silu_and_mul", lambda: ops.silu_and_mul(gu), gu.numel() * 2 * 3 // 2)
    # GEMMs: 1-SM (16 tokens, QKV), 2-SM gated gate_up (SiLU epilogue) and down_proj
    for name, m, n, kk, gated in (("gemm_1sm_qkv_m16", 16, 7168, H, False),
                                  ("gemm_2sm_gateup_silu", T, 2 * inter, H, True),
                                  ("gemm_2sm_down", T, H, inter, False)):
        wb = n * kk * 2
        nw = rot(lambda: torch.randn(n, kk, device=dev, dtype=bf) * 0.02, nrot(wb))
        xi = torch.randn(m, kk, device=dev, dtype=bf)
        add(name, (lambda nw=nw, xi=xi, gated=gated: ops.gate_up_silu(xi, nw()) if gated else ops.linear(xi, nw())),
            wb + xi.numel() * 2 + m * (n // 2 if gated else n) * 2)
    # sampling over the full vocabulary (fp32 logits)
    lg = rot(lambda: torch.randn(T, V, device=dev), 1 if small else 2)
    add("argmax", lambda: ops.argmax(lg()), T * V * 4)
    temp = torch.full((T,), 0.7, device=dev)
    tk = torch.full((T,), 50, device=dev, dtype=torch.int32)
    tp = torch.full((T,), 0.9, device=dev)
    seed = torch.arange(T, device=dev, dtype=torch.int64)
    step = torch.full((T,), 7, device=dev, dtype=torch.int64)
    add("sample_topk_topp", lambda: ops.sample(lg(), temp, tk, tp, seed, step), T * V * 4)
    # MoE decode (Qwen3-30B-A3B: hidden 2048, 128 experts of 768, top-8)
    from minisgl.ops.moe import moe_forward

    Hm, Im, E, topk = 2048, 768, 128, 8
    w1 = torch.randn(E, 2 * Im, Hm, device=dev, dtype=bf) * 0.02
    w2 = torch.randn(E, Hm, Im, device=dev, dtype=bf) * 0.02
    xm = torch.randn(T, Hm, device=dev, dtype=bf)
    gate = torch.randn(T, E, device=dev)
    ex = min(E, T * topk)  # experts touched (upper bound)
    add("moe_forward(route..combine)", lambda: moe_forward(xm, w1, w2, gate, topk, True, "silu"),
        ex * 3 * Im * Hm * 2)
    torch.cuda.synchronize()
    if a.once:
        print("ok", c.get_error())
        return
    hbm, _ = _peaks()
    print(f"suite bs={T}: kernel, us, GB/s (of measured HBM)")
    for name, us, gbs in rows:
        print(f"  {name:28s} {us:8.1f} us {gbs:8.0f} GB/s ({gbs * 1e9 / hbm:.2f})")
    print("ok", c.get_error())


def _gemm_sweep(a, c) -> None:
    """Decode GEMMs of Qwen3-14B at each TP degree's per-rank shapes: the automatic plan, every
    forced tiling (split count x 1-SM 128/256-row or 2-SM tiles) and cuBLAS (torch.matmul) on the
    same shape. One JSON line per (tp, shape, tokens): times in us, best forced variant, cuBLAS."""
    hbm, _ = _peaks()
    H, I, nq, nkv, hd = 5120, 17408, 40, 8, 128
    for tp in [int(t) for t in a.tps.split(",")]:
        kv = max(1, nkv // tp)
        shapes = {"qkv": ((nq // tp + 2 * kv) * hd, H, 0), "o": (H, nq * hd // tp, 0),
                  "gate_up": (2 * I // tp, H, 1), "down": (H, I // tp, 0)}
        for name, (N, K, epi) in shapes.items():
            nw = max(2, int(3e8 // (N * K * 2)) + 1)
            ws = [torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.02 for _ in range(nw)]
            wts = [w.t() for w in ws]
            for M in [int(m) for m in a.ms.split(",")]:
                x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
                out = torch.empty(M, N // 2 if epi == 1 else N, device="cuda", dtype=torch.bfloat16)
                it = [0]

                def ours(splits, wide):
                    def run():
                        c.gemm_ex(out, x, ws[it[0] % nw], None, epi, splits, wide)
                        it[0] += 1
                    return perf_cuda(run) * 1e3

                def cublas():
                    def run():
                        torch.matmul(x, wts[it[0] % nw])
                        it[0] += 1
                    return perf_cuda(run) * 1e3

                ours(-1, -1)  # warm the clocks and caches on this shape before timing anything
                row = {"tp": tp, "shape": name, "M": M, "N": N, "K": K}
                best = (1e9, None)
                bns = [-1] + ([64, 128] if M > 64 else [])  # token tiles: automatic, or several per batch
                for bn in bns:
                    c.gemm_force_bn(bn)
                    for wide in ([1, 2] if epi == 1 else [0, 1, 2]):
                        for splits in (1, 2, 3, 4, 6, 8):  # the tilings the GPU tests cover
                            if (wide == 2 and splits > 4) or (epi == 1 and splits > 4):
                                continue
                            try:
                                t = ours(splits, wide)
                            except RuntimeError:
                                continue
                            if t < best[0]:
                                best = (t, f"wide{wide}/s{splits}/bn{bn}")
                c.gemm_force_bn(-1)
                row["auto_us"] = round(ours(-1, -1), 2)
                row["best_us"], row["best"] = round(best[0], 2), best[1]
                row["cublas_us"] = round(cublas(), 2) if epi == 0 else None
                row["auto_hbm_frac"] = round(N * K * 2 / (row["auto_us"] * 1e-6) / hbm, 3)
                print(json.dumps(row), flush=True)
            del ws, wts
    print("ok", c.get_error())


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("op", choices=["gemm", "gemm-sweep", "decode-attn", "prefill-attn", "suite", "moe"])
    p.add_argument("--tps", default="1,2,4,8", help="gemm-sweep: TP degrees")
    p.add_argument("--ms", default="16,64,128,256", help="gemm-sweep: token counts")
    p.add_argument("--m", type=int, default=128)
    p.add_argument("--n", type=int, default=5120)
    p.add_argument("--k", type=int, default=5120)
    p.add_argument("--epi", type=int, default=0)
    p.add_argument("--bs", type=int, default=128)
    p.add_argument("--nq", type=int, default=40)
    p.add_argument("--nkv", type=int, default=8)
    p.add_argument("--tokens", type=int, default=16384)
    p.add_argument("--experts", type=int, default=128, help="moe: experts on this GPU")
    p.add_argument("--hidden", type=int, default=2880, help="moe: hidden size")
    p.add_argument("--inter", type=int, default=2880, help="moe: expert intermediate size")
    p.add_argument("--topk", type=int, default=4, help="moe: experts per token")
    p.add_argument("--impl", default="tcgen05", choices=["tcgen05", "mma", "trtllm"],
                   help="prefill-attn kernel (trtllm: FlashInfer's trtllm-gen kernel, for comparison)")
    p.add_argument("--once", action="store_true", help="run a few times untimed (for profilers)")
    p.add_argument("--trace", action="store_true", help="prefill-attn: per-CTA phase stamps of the tcgen05 kernel")
    p.add_argument("--trace-file", default=None, help="prefill-attn --trace: also save the raw stamps (.npy)")
    a = p.parse_args(argv)
    from minisgl._native import cuda

    c = cuda()
    {"gemm": _gemm, "gemm-sweep": _gemm_sweep, "decode-attn": _decode_attn, "prefill-attn": _prefill_attn, "moe": _moe,
     "suite": _suite}[a.op](a, c)


if __name__ == "__main__":
    main()
