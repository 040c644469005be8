"""Numerics of every sm_100a kernel against the plain PyTorch fp32 reference (ops/reference.py)."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

from minisgl.ops import reference as ref  # noqa: E402

DEV = "cuda"


def _c():
    from minisgl._native import cuda

    return cuda()


def _assert_no_device_error():
    code, info = _c().get_error()
    assert code == 0, f"device error {code} ({info})"


def _close(a, b, atol, rtol):
    torch.testing.assert_close(a.float().cpu(), b.float().cpu(), atol=atol, rtol=rtol)


@pytest.fixture(autouse=True)
def _cuda_only():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    torch.manual_seed(0)
    yield
    torch.cuda.synchronize()
    _assert_no_device_error()


def test_embedding():
    from minisgl import ops

    w = torch.randn(1000, 1024, device=DEV, dtype=torch.bfloat16)
    ids = torch.randint(0, 1000, (77,), device=DEV, dtype=torch.int32)
    _close(ops.embedding(w, ids), ref.embedding(w.cpu(), ids.cpu()), 0, 0)
    ids2 = torch.randint(0, 3000, (77,), device=DEV, dtype=torch.int32)
    _close(ops.embedding(w, ids2, 1000, 1000), ref.embedding(w.cpu(), ids2.cpu(), 1000, 1000), 0, 0)


@pytest.mark.parametrize("dim", [256, 1024, 5120, 2880])
def test_rmsnorm(dim):
    from minisgl import ops

    x = torch.randn(37, dim, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(dim, device=DEV, dtype=torch.bfloat16)
    _close(ops.rmsnorm(x, w, 1e-6), ref.rmsnorm(x.cpu().float(), w.cpu().float(), 1e-6), 2e-2, 2e-2)
    r = torch.randn_like(x)
    x1, r1 = x.clone(), r.clone()
    ops.fused_add_rmsnorm(x1, r1, w, 1e-6)
    x2, r2 = x.cpu().clone(), r.cpu().clone()
    ref.fused_add_rmsnorm(x2, r2, w.cpu(), 1e-6)
    _close(r1, r2, 0, 0)
    _close(x1, x2, 3e-2, 2e-2)


@pytest.mark.parametrize("M", [1, 7, 16, 33, 64, 100, 128, 200, 256, 300, 1000])
@pytest.mark.parametrize("N,K", [(256, 1024), (4096, 1024), (1024, 3072), (136, 200)])
def test_gemm(M, N, K):
    from minisgl import ops

    x = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=DEV, dtype=torch.bfloat16) / math.sqrt(K)
    y = ops.linear(x, w)
    torch.cuda.synchronize()
    expect = x.float() @ w.float().t()
    _close(y, expect, 3e-2, 2e-2)


@pytest.mark.parametrize("M", [3, 64, 256, 777])
def test_gemm_epilogues(M):
    from minisgl import ops

    K, N = 1024, 1024
    x = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=DEV, dtype=torch.bfloat16) / math.sqrt(K)
    b = torch.randn(N, device=DEV, dtype=torch.bfloat16)
    _close(ops.linear(x, w, b), x.float() @ w.float().t() + b.float(), 3e-2, 2e-2)
    out = torch.empty(M, N, device=DEV, dtype=torch.float32)
    _c().gemm(out, x, w, None, 3)
    _close(out, x.float() @ w.float().t(), 2e-3, 2e-3)
    y = ops.gate_up_silu(x, w)
    _close(y, ref.gate_up_silu(x.cpu().float(), w.cpu().float()), 3e-2, 3e-2)


def test_gemm_large_k_split():
    from minisgl import ops

    for M, N, K in [(8, 1024, 17408), (256, 5120, 5120), (1, 2048, 4096)]:
        x = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
        w = torch.randn(N, K, device=DEV, dtype=torch.bfloat16) / math.sqrt(K)
        for _ in range(2):  # second launch checks the split-K counters were re-armed
            _close(ops.linear(x, w), x.float() @ w.float().t(), 3e-2, 2e-2)


@pytest.mark.parametrize("hd,nq,nkv,norm", [(128, 16, 8, True), (64, 8, 2, False), (128, 40, 8, True)])
def test_qk_norm_rope_store(hd, nq, nkv, norm):
    from minisgl import ops

    T, slots = 50, 300
    qkv = torch.randn(T, (nq + 2 * nkv) * hd, device=DEV, dtype=torch.bfloat16)
    pos = torch.randint(0, 1000, (T,), device=DEV, dtype=torch.int32)
    cs = ref.rope_cos_sin(2048, hd, ref.default_inv_freq(hd, 1e6)).to(DEV)
    qn = torch.randn(hd, device=DEV, dtype=torch.bfloat16) if norm else None
    kn = torch.randn(hd, device=DEV, dtype=torch.bfloat16) if norm else None
    loc = torch.randperm(slots, device=DEV)[:T].to(torch.int32)
    kc = torch.zeros(slots, nkv, hd, device=DEV, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    q = ops.qk_norm_rope_store(qkv, pos, cs, qn, kn, 1e-6, kc, vc, loc, nq, nkv, hd)
    kc2, vc2 = kc.cpu().zero_(), vc.cpu().zero_()
    q2 = ref.qk_norm_rope_store(qkv.cpu(), pos.cpu(), cs.cpu(), None if qn is None else qn.cpu(),
                                None if kn is None else kn.cpu(), 1e-6, kc2, vc2, loc.cpu(), nq, nkv, hd)
    _close(q, q2, 3e-2, 3e-2)
    _close(kc, kc2, 3e-2, 3e-2)
    _close(vc, vc2, 0, 0)


def _paged_setup(lens_q, lens_kv, nq, nkv, hd, slots=4096, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    B = len(lens_kv)
    kc = torch.randn(slots, nkv, hd, generator=g).to(DEV, torch.bfloat16)
    vc = torch.randn(slots, nkv, hd, generator=g).to(DEV, torch.bfloat16)
    L = max(lens_kv)
    pt = torch.zeros(B + 3, (L + 31) // 32 * 32, dtype=torch.int32)
    perm = torch.randperm(slots, generator=g)
    used = 0
    rows = torch.arange(B, dtype=torch.int32) + 2  # rows are not 0..B-1
    for b, n in enumerate(lens_kv):
        pt[rows[b], :n] = perm[used : used + n].to(torch.int32)
        used += n
    cu = torch.zeros(B + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(torch.tensor(lens_q), 0)
    q = torch.randn(int(cu[-1]), nq, hd, generator=g).to(DEV, torch.bfloat16)
    return q, kc, vc, pt.to(DEV), rows.to(DEV), cu.to(DEV), torch.tensor(lens_kv, dtype=torch.int32, device=DEV)


@pytest.mark.parametrize("hd,nq,nkv", [(128, 16, 8), (128, 40, 8), (64, 64, 8), (128, 8, 8)])
@pytest.mark.parametrize("window,sinks", [(-1, False), (37, True)])
def test_attention_prefill(hd, nq, nkv, window, sinks):
    lens_q = [1, 17, 100, 64, 250]
    lens_kv = [1, 40, 100, 300, 250]  # prefix hits: kv longer than q
    q, kc, vc, pt, rows, cu, kvl = _paged_setup(lens_q, lens_kv, nq, nkv, hd)
    sk = torch.randn(nq, device=DEV) if sinks else None
    o = torch.empty_like(q)
    scale = 1 / math.sqrt(hd)
    _c().attention_prefill(o, q, kc, vc, pt, rows, cu, kvl, max(lens_q), scale, window, sk)
    e = ref.paged_attention(q.cpu(), kc.cpu(), vc.cpu(), pt.cpu(), rows.cpu(), cu.cpu(), kvl.cpu(), scale,
                            window, None if sk is None else sk.cpu())
    _close(o, e, 2e-2, 2e-2)


@pytest.mark.parametrize("hd,nq,nkv", [(128, 16, 8), (128, 40, 8), (64, 64, 8), (128, 64, 8)])
@pytest.mark.parametrize("splits", [1, 3, 8])
@pytest.mark.parametrize("window,sinks", [(-1, False), (128, True)])
def test_attention_decode(hd, nq, nkv, splits, window, sinks):
    lens_kv = [1, 5, 64, 65, 300, 1000, 777]
    B = len(lens_kv)
    q, kc, vc, pt, rows, cu, kvl = _paged_setup([1] * B, lens_kv, nq, nkv, hd)
    sk = torch.randn(nq, device=DEV) if sinks else None
    o = torch.empty_like(q)
    ws = torch.empty(B * nq * splits * (hd + 2) * 4, dtype=torch.uint8, device=DEV)
    scale = 1 / math.sqrt(hd)
    _c().attention_decode(o, q, kc, vc, pt, rows, kvl, scale, window, sk, splits, ws)
    e = ref.paged_attention(q.cpu(), kc.cpu(), vc.cpu(), pt.cpu(), rows.cpu(), cu.cpu(), kvl.cpu(), scale,
                            window, None if sk is None else sk.cpu())
    _close(o, e, 2e-2, 2e-2)


def _paged_pages_setup(lens_kv, nq, nkv, hd, page, seed=0):
    """Page-granular cache layout (what the engine allocates): each request owns whole pages of `page`
    consecutive slots, in shuffled page order; the page table stays token-granular."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    B = len(lens_kv)
    npages = sum((n + page - 1) // page for n in lens_kv) + 3
    slots = npages * page
    kc = torch.randn(slots, nkv, hd, generator=g).to(DEV, torch.bfloat16)
    vc = torch.randn(slots, nkv, hd, generator=g).to(DEV, torch.bfloat16)
    L = max(lens_kv)
    pt = torch.full((B + 3, (L + 63) // 64 * 64 + 64), 7, dtype=torch.int32)  # stale entries past the end
    perm = torch.randperm(npages, generator=g)
    used = 0
    rows = torch.arange(B, dtype=torch.int32) + 2
    for b, n in enumerate(lens_kv):
        for j in range((n + page - 1) // page):
            pt[rows[b], j * page : (j + 1) * page] = int(perm[used]) * page + torch.arange(page, dtype=torch.int32)
            used += 1
    q = torch.randn(B, nq, hd, generator=g).to(DEV, torch.bfloat16)
    cu = torch.arange(B + 1, dtype=torch.int32)
    return q, kc, vc, pt.to(DEV), rows.to(DEV), cu.to(DEV), torch.tensor(lens_kv, dtype=torch.int32, device=DEV)


@pytest.mark.parametrize("hd,nq,nkv", [(128, 40, 8), (64, 64, 8), (128, 8, 8), (128, 16, 1)])
@pytest.mark.parametrize("page", [16, 32, 64])
@pytest.mark.parametrize("window,sinks", [(-1, False), (100, True)])
@pytest.mark.parametrize("num_ctas", [148, 3])
def test_attention_decode_paged(hd, nq, nkv, page, window, sinks, num_ctas):
    """Persistent paged decode (work list, TMA page loads, last-arriver combine) against the fp32
    reference; few CTAs force multi-chunk requests; run twice to check the counters return to zero."""
    _paged_decode_case(hd, nq, nkv, page, window, sinks, num_ctas, [1, 5, 64, 65, 300, 1000, 777, 4000, 129])


@pytest.mark.parametrize("page", [16, 64])
@pytest.mark.parametrize("num_ctas", [148, 2])
def test_attention_decode_paged_short_window(page, num_ctas):
    """gpt-oss-style decode: head_dim 64, 2 query heads per kv head, a 16-token sliding window and
    sinks, on requests around the window length (every kv length from 1 to 48)."""
    _paged_decode_case(64, 4, 2, page, 16, True, num_ctas, list(range(1, 49)))


def _paged_decode_case(hd, nq, nkv, page, window, sinks, num_ctas, lens_kv):
    from minisgl.attention.paged import decode_work_list
    import numpy as np

    B = len(lens_kv)
    q, kc, vc, pt, rows, cu, kvl = _paged_pages_setup(lens_kv, nq, nkv, hd, page)
    sk = torch.randn(nq, device=DEV) if sinks else None
    work, n = decode_work_list(np.array(lens_kv), nkv, num_ctas)
    work_d = torch.from_numpy(work).to(DEV)
    n_d = torch.tensor([n], dtype=torch.int32, device=DEV)
    G = nq // nkv
    ws = torch.empty(n * nkv * G * (hd + 2), dtype=torch.float32, device=DEV)
    counters = torch.zeros(B * nkv, dtype=torch.int32, device=DEV)
    scale = 1 / math.sqrt(hd)
    e = ref.paged_attention(q.cpu(), kc.cpu(), vc.cpu(), pt.cpu(), rows.cpu(), cu.cpu(), kvl.cpu(), scale,
                            window, None if sk is None else sk.cpu())
    for _ in range(2):
        o = torch.full_like(q, float("nan"))
        _c().attention_decode_paged(o, q, kc, vc, pt, rows, kvl, work_d, n_d, ws, n, counters, scale, window, sk,
                                    page)
        _close(o, e, 2e-2, 2e-2)
        assert int(counters.abs().sum()) == 0
    assert _c().get_error() == (0, 0)


@pytest.mark.parametrize("nq,nkv", [(40, 8), (64, 8), (8, 8), (32, 2)])
@pytest.mark.parametrize("page", [16, 32, 64])
@pytest.mark.parametrize("window,sinks", [(-1, False), (100, True)])
def test_attention_prefill_tcgen05(nq, nkv, page, window, sinks, qscale=2.0):
    """tcgen05 prefill attention (S / O in TMEM, MN-major V operand, lazy O rescaling, two softmax
    warps per row split by keys) against the fp32 reference: ragged requests, prefix hits (kv
    longer than q), partial last tiles."""
    hd = 128
    lens_q = [1, 17, 300, 64, 129, 700]
    lens_kv = [1, 40, 300, 400, 129, 1000]
    _, kc, vc, pt, rows, _, kvl = _paged_pages_setup(lens_kv, nq, nkv, hd, page, seed=3)
    g = torch.Generator(device="cpu").manual_seed(4)
    q = (torch.randn(sum(lens_q), nq, hd, generator=g) * qscale).to(DEV, torch.bfloat16)
    cu = torch.zeros(len(lens_q) + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(torch.tensor(lens_q), 0)
    cu = cu.to(DEV)
    sk = torch.randn(nq, device=DEV) if sinks else None
    o = torch.full_like(q, float("nan"))
    scale = 1 / math.sqrt(hd)
    _c().attention_prefill_fmha(o, q, kc, vc, pt, rows, cu, kvl, max(lens_q), scale, window, sk, page)
    e = ref.paged_attention(q.cpu(), kc.cpu(), vc.cpu(), pt.cpu(), rows.cpu(), cu.cpu(), kvl.cpu(), scale, window,
                            None if sk is None else sk.cpu())
    _close(o, e, 2e-2, 2e-2)
    assert _c().get_error() == (0, 0)



@pytest.mark.parametrize("window", [-1, 300])
def test_attention_prefill_tcgen05_peaked_scores(window):
    """Large query norms: row maxima jump by far more than the lazy-rescale threshold from block
    to block, so O is rescaled in TMEM on most blocks."""
    test_attention_prefill_tcgen05(40, 8, 64, window, False, qscale=8.0)

def test_argmax_and_greedy_sample():
    from minisgl import ops

    logits = torch.randn(33, 151936, device=DEV)
    logits[3, 5] = logits[3, 9] = 100.0  # tie -> lowest index
    assert torch.equal(ops.argmax(logits).cpu(), ref.argmax(logits.cpu()))
    assert torch.equal(ops.argmax(logits.bfloat16()).cpu(), ref.argmax(logits.bfloat16().cpu()))
    # shard form: first `vocab` columns, with the maxima (what vocab-parallel greedy sampling exchanges)
    for v in (151936, 75968, 75965, 37):
        idx, val = ops.argmax(logits, vocab=v, with_values=True)
        ev, ei = logits[:, :v].cpu().max(dim=-1)
        assert torch.equal(idx.cpu(), ei.to(torch.int32)), v
        assert torch.equal(val.cpu(), ev), v
    # an unaligned row start takes the scalar path
    sub = logits[:, 1:]
    assert torch.equal(ops.argmax(sub).cpu(), ref.argmax(sub.cpu()))


def test_sampling_matches_reference():
    from minisgl import ops

    B, V = 16, 5000
    logits = torch.randn(B, V, device=DEV) * 3
    temp = torch.tensor([0.0, 0.7, 1.0, 1.3] * 4, device=DEV)
    topk = torch.tensor([V, 1, 50, V] * 4, dtype=torch.int32, device=DEV)
    topp = torch.tensor([1.0, 1.0, 0.9, 0.5] * 4, device=DEV)
    seed = torch.arange(B, dtype=torch.int64, device=DEV) * 7 + 1
    step = torch.arange(B, dtype=torch.int64, device=DEV) + 100
    a = ops.sample(logits, temp, topk, topp, seed, step).cpu()
    b = ref.sample(logits.cpu(), temp.cpu(), topk.cpu(), topp.cpu(), seed.cpu(), step.cpu())
    assert (a == b).float().mean() >= 0.9, (a, b)
    # kept-set property: every draw lies inside its top-k
    for i in range(B):
        k = int(topk[i])
        if 0 < k < V:
            kth = torch.topk(logits[i].cpu() / max(float(temp[i]), 1e-6), k).values[-1]
            assert logits[i, a[i]].cpu() / max(float(temp[i]), 1e-6) >= kth


@pytest.mark.parametrize("case", ["topk_fast", "topk_full", "topp_only", "temp_only", "tie_overflow"])
def test_sampling_paths(case):
    """Each path of the sampling kernel on a full-size vocabulary: top-k <= 4096 (shared-memory
    candidate list), larger top-k (whole-row passes), top-p alone, temperature alone, and a row of
    ties at the top-k threshold that overflows the candidate list. Every draw must lie in the kept
    set (top-k by the float threshold, then the top-p nucleus up to float rounding at its edge);
    draws agree with the fp32/fp64 reference and are deterministic."""
    from minisgl import ops

    B, V = 24, 151936
    g = torch.Generator(device="cpu").manual_seed(7)
    logits = torch.randn(B, V, generator=g) * 2
    k, p = {"topk_fast": (40, 0.9), "topk_full": (6000, 0.95), "topp_only": (V, 0.8), "temp_only": (V, 1.0),
            "tie_overflow": (10, 1.0)}[case]
    if case == "tie_overflow":
        logits[:, :5000] = 3.0  # 5000 tokens tie at the 10th-largest value
        logits[:, 5000:] = torch.randn(B, V - 5000, generator=g).clamp(max=2.5)
    temp = torch.full((B,), 0.8)
    topk = torch.full((B,), k, dtype=torch.int32)
    topp = torch.full((B,), p)
    seed = torch.arange(B, dtype=torch.int64) * 13 + 5
    step = torch.arange(B, dtype=torch.int64) + 40
    args = [x.to(DEV) for x in (temp, topk, topp, seed, step)]
    a = ops.sample(logits.to(DEV), *args).cpu()
    a2 = ops.sample(logits.to(DEV), *args).cpu()
    assert torch.equal(a, a2)
    b = ref.sample(logits, temp, topk, topp, seed, step)
    assert (a == b).float().mean() >= 0.9, (a, b)
    for i in range(B):
        z = logits[i] / 0.8
        keep = torch.ones(V, dtype=torch.bool)
        if 0 < k < V:
            keep &= z >= torch.topk(z, k).values[-1]
        assert keep[a[i]], (i, int(a[i]))
        if p < 1.0:
            pr = torch.softmax(z.double().masked_fill(~keep, float("-inf")), -1)
            above = pr[pr > pr[a[i]]].sum()  # mass strictly above the drawn token
            assert above < p + 1e-4, (i, float(above))


@pytest.mark.parametrize("tp", [2, 8])
def test_sampling_shards_reproduce_unsharded_draws(tp):
    """What vocabulary-parallel sampling does on each rank, emulated on one GPU: (1) temperature-only
    and greedy rows drawn per shard (token ids offset, winning scores returned) and combined by best
    score equal the unsharded draw; (2) top-k rows sampled over gathered per-shard candidate lists
    (sorted by token id, passed as column ids) equal the unsharded draw."""
    from minisgl import ops

    B, V = 32, 151936
    g = torch.Generator(device="cpu").manual_seed(11)
    logits = (torch.randn(B, V, generator=g) * 2).to(DEV)
    seed = (torch.arange(B, dtype=torch.int64) * 7 + 3).to(DEV)
    step = (torch.arange(B, dtype=torch.int64) + 17).to(DEV)
    width = (V + tp - 1) // tp
    shards = [(r * width, min(V, (r + 1) * width)) for r in range(tp)]
    # (1) temperature only, every other row greedy
    temp = torch.tensor([0.0 if i % 2 else 0.9 for i in range(B)], device=DEV)
    k = torch.full((B,), V, dtype=torch.int32, device=DEV)
    p = torch.ones(B, device=DEV)
    want = ops.sample(logits, temp, k, p, seed, step)
    ids, vals = zip(*[ops.sample(logits[:, lo:hi].contiguous(), temp, k, p, seed, step, id_offset=lo,
                                 with_values=True) for lo, hi in shards])
    best = torch.stack(vals).argmax(0)
    got = torch.stack(ids).gather(0, best.view(1, B)).view(B)
    assert torch.equal(got.cpu(), want.cpu())
    # (2) top-k 40 (every third row also top-p 0.9) from per-shard candidate lists
    temp = torch.full((B,), 0.8, device=DEV)
    k = torch.full((B,), 40, dtype=torch.int32, device=DEV)
    p = torch.tensor([0.9 if i % 3 == 0 else 1.0 for i in range(B)], device=DEV)
    want = ops.sample(logits, temp, k, p, seed, step).cpu()
    cv, ci = [], []
    for lo, hi in shards:
        v, i = torch.topk(logits[:, lo:hi], 56, dim=1)
        cv.append(v)
        ci.append(i.to(torch.int32) + lo)
    cid, order = torch.sort(torch.cat(ci, 1), dim=1)
    cval = torch.cat(cv, 1).gather(1, order).contiguous()
    got = ops.sample(cval, temp, k, p, seed, step, col_ids=cid.contiguous()).cpu()
    exact = p.cpu() >= 1.0
    assert torch.equal(got[exact], want[exact])
    assert (got == want).float().mean() >= 0.9


def test_store_kv():
    from minisgl import ops

    k = torch.randn(20, 8 * 128, device=DEV, dtype=torch.bfloat16)
    v = torch.randn_like(k)
    kc = torch.zeros(100, 8, 128, device=DEV, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    loc = torch.randperm(100, device=DEV)[:20].to(torch.int32)
    ops.store_kv(k, v, kc, vc, loc)
    kc2, vc2 = kc.cpu().zero_(), vc.cpu().zero_()
    ref.store_kv(k.cpu(), v.cpu(), kc2, vc2, loc.cpu())
    _close(kc, kc2, 0, 0)
    _close(vc, vc2, 0, 0)


@pytest.mark.parametrize("M", [5, 130, 190, 220, 256, 600])
@pytest.mark.parametrize("epi", [0, 1, 3])
@pytest.mark.parametrize("wide,splits", [(0, 1), (1, 1), (0, 3), (1, 4), (-1, -1), (2, 1), (2, 2), (2, 3)])
@pytest.mark.parametrize("blocked", [False, True])
def test_gemm_variants(M, epi, wide, splits, blocked):
    """Every tiling (128/256-row weight tiles, 2-SM pairs (wide=2) with 64..256-token tiles, forced split-K with
    the cluster exchange) against the fp32 reference, run twice, with bias."""
    K, N = 1536, 768
    x = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=DEV, dtype=torch.bfloat16) / math.sqrt(K)
    b = torch.randn(N, device=DEV, dtype=torch.bfloat16)
    if epi == 1:
        expect = ref.gate_up_act(x.cpu().float() @ w.cpu().float().t() + b.cpu().float())
        out = torch.empty(M, N // 2, device=DEV, dtype=torch.bfloat16)
    else:
        expect = x.cpu().float() @ w.cpu().float().t() + b.cpu().float()
        out = torch.empty(M, N, device=DEV, dtype=torch.float32 if epi == 3 else torch.bfloat16)
    wk = w.view(N, K // 64, 64).transpose(0, 1).contiguous() if blocked else w
    for _ in range(2):
        out.zero_()
        _c().gemm_ex(out, x, wk, b, epi, splits, wide)
        _close(out, expect, 3e-2, 3e-2)


@pytest.mark.parametrize("T,E,topk,H,I,act,renorm,after,bias", [
    (1, 8, 2, 256, 128, "silu", True, False, False),
    (37, 8, 2, 256, 128, "silu", True, False, False),
    (300, 64, 8, 1024, 384, "silu", True, False, False),
    (64, 32, 4, 512, 360, "swiglu_oai", False, True, True),
    (513, 128, 4, 2880, 360, "swiglu_oai", False, True, True),
])
def test_moe_forward(T, E, topk, H, I, act, renorm, after, bias):
    from minisgl.moe.grouped import moe_reference
    from minisgl.ops.moe import moe_forward

    g = torch.Generator().manual_seed(T + E)
    x = torch.randn(T, H, generator=g).to(DEV, torch.bfloat16)
    w1 = (torch.randn(E, 2 * I, H, generator=g) / math.sqrt(H)).to(DEV, torch.bfloat16)
    w2 = (torch.randn(E, H, I, generator=g) / math.sqrt(I)).to(DEV, torch.bfloat16)
    gate = torch.randn(T, E, generator=g).to(DEV)
    b1 = (torch.randn(E, 2 * I, generator=g) * 0.1).to(DEV, torch.bfloat16) if bias else None
    b2 = (torch.randn(E, H, generator=g) * 0.1).to(DEV, torch.bfloat16) if bias else None
    out = moe_forward(x, w1, w2, gate, topk, renorm, act, b1, b2, after)
    exp = moe_reference(x.cpu(), w1.cpu(), w2.cpu(), gate.cpu(), topk, renorm, act,
                        None if b1 is None else b1.cpu(), None if b2 is None else b2.cpu(), after)
    _close(out, exp, 3e-2, 3e-2)
    # the activation in the first grouped GEMM's epilogue (gate/up interleaved, I padded to 128)
    from minisgl.ops.moe import interleave_experts

    w1i, w2i, b1i = interleave_experts(w1, w2, b1)
    out = moe_forward(x, w1i, w2i, gate, topk, renorm, act, b1i, b2, after, w1_interleaved=True)
    _close(out, exp, 3e-2, 3e-2)
    # expert parallelism: this "rank" holds experts [E/4, E/2); assignments elsewhere drop out
    e0, n = E // 4, E // 4
    sub = lambda t: None if t is None else t[e0 : e0 + n].contiguous()
    out = moe_forward(x, sub(w1), sub(w2), gate, topk, renorm, act, sub(b1), sub(b2), after, expert_offset=e0)
    exp = moe_reference(x.cpu(), sub(w1).cpu(), sub(w2).cpu(), gate.cpu(), topk, renorm, act,
                        None if b1 is None else sub(b1).cpu(), None if b2 is None else sub(b2).cpu(), after,
                        expert_offset=e0)
    _close(out, exp, 3e-2, 3e-2)


@pytest.mark.parametrize("n_tok,n_writes", [(1, 1), (256, 256), (5000, 5064), (16384, 16384)])
def test_plan_apply_gather_scatter(n_tok, n_writes):
    """Batch metadata kernel: page-table writes then the out_loc gather (which must see them), and
    the int32 gather / scatter of decode input ids and sampled tokens, against torch indexing."""
    g = torch.Generator(device="cpu").manual_seed(n_tok)
    rows, cols = 300, 4096
    pt = torch.randint(0, 1 << 20, (rows, cols), generator=g, dtype=torch.int32)
    # distinct (row, pos) write targets; the tokens read some of them and some untouched entries
    flat = torch.randperm(rows * cols, generator=g)[:n_writes]
    pt_rows, pt_pos = (flat // cols).to(torch.int32), (flat % cols).to(torch.int32)
    pt_slots = torch.randint(0, 1 << 20, (n_writes,), generator=g, dtype=torch.int32)
    pick = torch.randint(0, rows * cols, (n_tok,), generator=g)
    pick[: n_tok // 2] = flat[torch.randint(0, n_writes, (n_tok // 2,), generator=g)]
    tok_rows, positions = (pick // cols).to(torch.int32), (pick % cols).to(torch.int32)
    exp_pt = pt.clone()
    exp_pt[pt_rows.long(), pt_pos.long()] = pt_slots
    exp_loc = exp_pt[tok_rows.long(), positions.long()]
    dpt = pt.to(DEV)
    out_loc = torch.empty(n_tok, dtype=torch.int32, device=DEV)
    _c().plan_apply(dpt, pt_rows.to(DEV), pt_pos.to(DEV), pt_slots.to(DEV), tok_rows.to(DEV), positions.to(DEV),
                    out_loc)
    assert torch.equal(dpt.cpu(), exp_pt)
    assert torch.equal(out_loc.cpu(), exp_loc)
    src = torch.randint(-1000, 1000, (rows + 2,), generator=g, dtype=torch.int32)
    idx = torch.randint(0, rows + 2, (n_tok,), generator=g, dtype=torch.int32)
    dst = torch.empty(n_tok, dtype=torch.int32, device=DEV)
    _c().gather_i32(dst, src.to(DEV), idx.to(DEV))
    assert torch.equal(dst.cpu(), src[idx.long()])
    uniq = torch.randperm(rows + 2, generator=g)[: min(n_tok, rows + 2)].to(torch.int32)
    vals = torch.randint(-1000, 1000, (uniq.numel(),), generator=g, dtype=torch.int32)
    sc = src.to(DEV)
    _c().scatter_i32(sc, uniq.to(DEV), vals.to(DEV))
    exp = src.clone()
    exp[uniq.long()] = vals
    assert torch.equal(sc.cpu(), exp)


@pytest.mark.parametrize("M", [1, 7, 64, 130, 256])
@pytest.mark.parametrize("N,n_valid,K", [(1024, 1001, 256), (18992, 18992, 5120), (151936, 151936, 1024)])
def test_lm_head_argmax(M, N, n_valid, K):
    """Greedy pick fused into the LM-head GEMM (no logits written) against the argmax of the fp32
    logits over the first n_valid rows: the same id wherever the best logit leads the second by more
    than the GEMM's bf16-input rounding, and a maximum within that rounding of the true one."""
    g = torch.Generator(device="cpu").manual_seed(M + N)
    x = torch.randn(M, K, generator=g).to(DEV, torch.bfloat16)
    w = (torch.randn(N, K, generator=g) / math.sqrt(K)).to(DEV, torch.bfloat16)
    w[n_valid:] = 10.0  # padding rows must never win
    bias = (torch.randn(N, generator=g) * 0.1).to(DEV, torch.bfloat16) if N == 1024 else None
    ids = torch.empty(M, dtype=torch.int32, device=DEV)
    vals = torch.empty(M, dtype=torch.float32, device=DEV)
    _c().lm_head_argmax(ids, vals, x, w, bias, n_valid, 5)
    logits = x.float() @ w[:n_valid].float().t()
    if bias is not None:
        logits += bias[:n_valid].float()
    top2 = torch.topk(logits, 2, dim=1).values
    exp = logits.argmax(dim=1).to(torch.int32) + 5
    clear = (top2[:, 0] - top2[:, 1]) > 1e-3
    assert torch.equal(ids[clear].cpu(), exp[clear].cpu())
    got = logits.gather(1, (ids.long() - 5).clamp(0, n_valid - 1)[:, None])[:, 0]
    torch.testing.assert_close(got.cpu(), top2[:, 0].cpu(), atol=1e-3, rtol=1e-4)
    torch.testing.assert_close(vals.cpu(), top2[:, 0].cpu(), atol=1e-3, rtol=1e-4)


@pytest.mark.parametrize("M", [100, 256])
@pytest.mark.parametrize("bn", [64, 128, 256])
@pytest.mark.parametrize("wide,splits", [(0, 1), (0, 2), (0, 6), (0, 8), (1, 3), (2, 1), (2, 4)])
def test_gemm_token_tiles(M, bn, wide, splits):
    """Token-tile overrides (several token tiles per weight tile) with split-K up to 8-CTA clusters:
    the tilings a tiling sweep may pick, against the fp32 reference."""
    K, N = 1536, 768
    x = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=DEV, dtype=torch.bfloat16) / math.sqrt(K)
    expect = x.cpu().float() @ w.cpu().float().t()
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    try:
        _c().gemm_force_bn(bn)
        for _ in range(2):
            out.zero_()
            _c().gemm_ex(out, x, w, None, 0, splits, wide)
            _close(out, expect, 3e-2, 3e-2)
    finally:
        _c().gemm_force_bn(-1)


@pytest.mark.parametrize("T", [5, 64, 300])
@pytest.mark.parametrize("H,inter,act,bias", [(512, 384, "swiglu_oai", True), (2880, 256, "silu", False)])
def test_moe_mxfp4_experts_match_dequantised(T, H, inter, act, bias):
    """MoE forward with MXFP4 experts kept in fp4 (the grouped GEMM converts each tile to bf16 in
    shared memory) equals the bf16 path on the dequantised weights bit for bit (power-of-two scales
    make the conversion exact; the MMA sequence is the same), and the fp32 reference within bf16
    tolerance. H = 2880 leaves a partial last 128-row tile of the down projection."""
    from minisgl.moe.grouped import moe_reference
    from minisgl.moe.mxfp4 import Mxfp4Experts, dequant_mxfp4, interleave_rows, pad_k
    from minisgl.ops.moe import interleave_experts, moe_forward

    E, topk = 8, 4
    g = torch.Generator().manual_seed(T + H)
    b1 = torch.randint(0, 256, (E, 2 * inter, H // 32, 16), generator=g, dtype=torch.int32).to(torch.uint8)
    s1 = torch.randint(116, 120, (E, 2 * inter, H // 32), generator=g, dtype=torch.int32).to(torch.uint8)
    b2 = torch.randint(0, 256, (E, H, inter // 32, 16), generator=g, dtype=torch.int32).to(torch.uint8)
    s2 = torch.randint(116, 120, (E, H, inter // 32), generator=g, dtype=torch.int32).to(torch.uint8)
    bias1 = (torch.randn(E, 2 * inter, generator=g) * 0.1).to(DEV, torch.bfloat16) if bias else None
    bias2 = (torch.randn(E, H, generator=g) * 0.1).to(DEV, torch.bfloat16) if bias else None
    x = (torch.randn(T, H, generator=g)).to(DEV, torch.bfloat16)
    gating = torch.randn(T, E, generator=g).to(DEV)
    w1 = dequant_mxfp4(b1, s1, torch.bfloat16).to(DEV)
    w2 = dequant_mxfp4(b2, s2, torch.bfloat16).to(DEV)
    w1i, w2i, b1i = interleave_experts(w1, w2, bias1)
    ip = w1i.shape[1] // 2
    q1 = Mxfp4Experts.pack(interleave_rows(b1.to(DEV)), interleave_rows(s1.to(DEV)), 256)
    q2 = Mxfp4Experts.pack(*pad_k(b2.to(DEV), s2.to(DEV), ip), 128)
    soft_after = act == "swiglu_oai"
    ref16 = moe_forward(x, w1i, w2i, gating, topk, True, act, b1i, bias2, soft_after, 0, True)
    out = moe_forward(x, q1, q2, gating, topk, True, act, b1i, bias2, soft_after, 0, True)
    torch.cuda.synchronize()
    assert _c().get_error() == (0, 0)
    assert torch.equal(out, ref16)
    ref = moe_reference(x.cpu().float(), w1.cpu().float(), w2.cpu().float(), gating.cpu(), topk, True, act,
                        None if bias1 is None else bias1.cpu().float(), None if bias2 is None else bias2.cpu().float(),
                        soft_after)
    # bf16 activations between the two GEMMs: errors scale with the output's range
    tol = 2e-2 * float(ref.abs().max())
    _close(out, ref.to(DEV), tol, 2e-2)
