"""The bounds-check kernel build (``minisgl._cuda_bc``, loaded with ``MINISGL_BOUNDS_CHECK=1``).

Each test hands one kernel an index just past the end of its table and expects the build to record
(kErrBounds = 3, site) in the device error word and skip the access. Every table is a view of a
larger allocation, so that even a missed check would touch only memory this test owns: none of
these launches can fault the GPU. Valid inputs must give the release build's results bit for bit.
"""

import importlib
import math
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BOUNDS = 3
SITE_EMBED, SITE_SLOT, SITE_POS, SITE_ROW, SITE_ATTN_SLOT, SITE_PERM, SITE_INV = 1, 2, 3, 4, 5, 6, 7


@pytest.fixture(scope="module")
def bc():
    import minisgl._cuda  # noqa: F401  (loads libtorch's CUDA pieces first)

    m = importlib.import_module("minisgl._cuda_bc")
    m.get_error()
    return m


@pytest.fixture(scope="module")
def rel():
    m = importlib.import_module("minisgl._cuda")
    m.get_error()
    return m


def _err(m):
    torch.cuda.synchronize()
    return tuple(m.get_error())


def test_embedding_id_out_of_vocab(bc, rel):
    V, H = 100, 256
    big = torch.randn(V + 8, H, device=DEV).bfloat16()
    w = big[:V]
    ids = torch.tensor([3, V, 7], dtype=torch.int32, device=DEV)
    out = torch.empty(3, H, device=DEV, dtype=torch.bfloat16)
    bc.embedding(out, w, ids, 0, V, False)
    assert _err(bc) == (BOUNDS, SITE_EMBED)
    ok = torch.tensor([3, 9, 7], dtype=torch.int32, device=DEV)
    o1, o2 = torch.empty_like(out), torch.empty_like(out)
    bc.embedding(o1, w, ok, 0, V, False)
    rel.embedding(o2, w, ok, 0, V, False)
    assert _err(bc) == (0, 0) and torch.equal(o1, o2)


def test_store_kv_slot_out_of_cache(bc):
    S, nkv, hd = 64, 2, 128
    bigk = torch.zeros(S + 8, nkv, hd, device=DEV, dtype=torch.bfloat16)
    bigv = torch.zeros_like(bigk)
    k = torch.randn(3, nkv * hd, device=DEV).bfloat16()
    v = torch.randn(3, nkv * hd, device=DEV).bfloat16()
    loc = torch.tensor([1, S, 5], dtype=torch.int32, device=DEV)
    bc.store_kv(k, v, bigk[:S], bigv[:S], loc)
    assert _err(bc) == (BOUNDS, SITE_SLOT)
    assert int(bigk[S:].abs().sum()) == 0 and int(bigv[S:].abs().sum()) == 0  # skipped, not written
    assert torch.equal(bigk[1].reshape(-1), k[0]) and torch.equal(bigk[5].reshape(-1), k[2])


def test_rope_position_and_slot(bc, rel):
    nq, nkv, hd, T, S, P = 4, 2, 128, 3, 32, 16
    qkv = torch.randn(T, (nq + 2 * nkv) * hd, device=DEV).bfloat16()
    bigcs = torch.randn(P + 8, hd, device=DEV)
    cs = bigcs[:P]
    kc = torch.zeros(S + 8, nkv, hd, device=DEV, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    q = torch.empty(T, nq, hd, device=DEV, dtype=torch.bfloat16)
    pos = torch.tensor([0, P, 2], dtype=torch.int32, device=DEV)
    loc = torch.tensor([0, 1, 2], dtype=torch.int32, device=DEV)
    bc.qk_norm_rope_store(q, qkv, pos, cs, None, None, 1e-6, kc[:S], vc[:S], loc, nq, nkv, hd)
    assert _err(bc) == (BOUNDS, SITE_POS)
    pos = torch.tensor([0, 1, 2], dtype=torch.int32, device=DEV)
    loc = torch.tensor([0, S, 2], dtype=torch.int32, device=DEV)
    bc.qk_norm_rope_store(q, qkv, pos, cs, None, None, 1e-6, kc[:S], vc[:S], loc, nq, nkv, hd)
    assert _err(bc) == (BOUNDS, SITE_SLOT)
    assert int(kc[S:].abs().sum()) == 0 and int(vc[S:].abs().sum()) == 0
    # valid inputs: same bits as the release build
    loc = torch.tensor([3, 4, 5], dtype=torch.int32, device=DEV)
    q1, q2 = torch.empty_like(q), torch.empty_like(q)
    k1, k2 = torch.zeros_like(kc), torch.zeros_like(kc)
    v1, v2 = torch.zeros_like(kc), torch.zeros_like(kc)
    bc.qk_norm_rope_store(q1, qkv, pos, cs, None, None, 1e-6, k1[:S], v1[:S], loc, nq, nkv, hd)
    rel.qk_norm_rope_store(q2, qkv, pos, cs, None, None, 1e-6, k2[:S], v2[:S], loc, nq, nkv, hd)
    assert _err(bc) == (0, 0)
    assert torch.equal(q1, q2) and torch.equal(k1, k2) and torch.equal(v1, v2)


def _pages(lens, nq, nkv, hd, page, extra_rows=2):
    """Page-granular cache (views of larger tensors) and a token page table with spare rows after
    the used ones, so an over-long kv length still reads inside the table's allocation."""
    g = torch.Generator().manual_seed(0)
    npages = sum((n + page - 1) // page for n in lens) + 2
    S = npages * page
    bigk = torch.randn(S + 2 * page, nkv, hd, generator=g).to(DEV, torch.bfloat16)
    bigv = torch.randn(S + 2 * page, nkv, hd, generator=g).to(DEV, torch.bfloat16)
    stride = (max(lens) + 63) // 64 * 64 + 64
    pt = torch.zeros(len(lens) + extra_rows, stride, dtype=torch.int32)
    k = 0
    for b, n in enumerate(lens):
        for j in range((n + page - 1) // page):
            pt[b, j * page:(j + 1) * page] = k * page + torch.arange(page, dtype=torch.int32)
            k += 1
    rows = torch.arange(len(lens), dtype=torch.int32)
    q = torch.randn(len(lens), nq, hd, generator=g).to(DEV, torch.bfloat16)
    return q, bigk, bigv, S, pt, rows, stride


@pytest.mark.parametrize("kind", ["mma", "paged"])
def test_decode_attention_page_table_checks(bc, rel, kind):
    from minisgl.attention.paged import decode_work_list

    nq, nkv, hd, page = 16, 2, 128, 16
    lens = [40, 100, 17]
    q, bigk, bigv, S, pt, rows, stride = _pages(lens, nq, nkv, hd, page)
    kc, vc = bigk[:S], bigv[:S]
    scale = 1 / math.sqrt(hd)

    def run(m, pt_h, lens_h):
        o = torch.zeros_like(q)
        ptd, kvl = pt_h.to(DEV), torch.tensor(lens_h, dtype=torch.int32, device=DEV)
        if kind == "mma":
            ws = torch.empty(len(lens_h) * nq * 2 * (hd + 2) * 4, dtype=torch.uint8, device=DEV)
            m.attention_decode(o, q, kc, vc, ptd[: len(lens_h)], rows.to(DEV), kvl, scale, -1, None, 2, ws)
        else:
            work, n = decode_work_list(np.array(lens_h), nkv, 4)
            ws = torch.empty(n * nq * (hd + 2), dtype=torch.float32, device=DEV)
            cnt = torch.zeros(len(lens_h) * nkv, dtype=torch.int32, device=DEV)
            m.attention_decode_paged(o, q, kc, vc, ptd[: len(lens_h)], rows.to(DEV), kvl,
                                     torch.from_numpy(work).to(DEV), torch.tensor([n], dtype=torch.int32, device=DEV),
                                     ws, n, cnt, scale, -1, None, page)
        return o

    o1, o2 = run(bc, pt, lens), run(rel, pt, lens)
    assert _err(bc) == (0, 0) and torch.equal(o1, o2)
    bad = pt.clone()
    bad[1, 32:48] = S + torch.arange(page, dtype=torch.int32)  # a page past the cache
    run(bc, bad, lens)
    assert _err(bc) == (BOUNDS, SITE_ATTN_SLOT)
    run(bc, pt, [40, stride + 16, 17])  # kv length past the page-table row
    assert _err(bc) == (BOUNDS, SITE_ROW)


def test_prefill_attention_page_table_checks(bc, rel):
    nq, nkv, hd, page = 16, 2, 128, 16
    lens = [40, 100, 17]
    _, bigk, bigv, S, pt, rows, stride = _pages(lens, nq, nkv, hd, page)
    kc, vc = bigk[:S], bigv[:S]
    g = torch.Generator().manual_seed(1)
    q = torch.randn(sum(lens), nq, hd, generator=g).to(DEV, torch.bfloat16)
    cu = torch.tensor([0] + np.cumsum(lens).tolist(), dtype=torch.int32, device=DEV)
    scale = 1 / math.sqrt(hd)

    def run(m, pt_h, lens_kv, fmha):
        o = torch.zeros_like(q)
        ptd, kvl, r = pt_h.to(DEV), torch.tensor(lens_kv, dtype=torch.int32, device=DEV), rows.to(DEV)
        if fmha:
            m.attention_prefill_fmha(o, q, kc, vc, ptd[:3], r, cu, kvl, max(lens), scale, -1, None, page)
        else:
            m.attention_prefill(o, q, kc, vc, ptd[:3], r, cu, kvl, max(lens), scale, -1, None)
        return o

    for fmha in (False, True):
        o1, o2 = run(bc, pt, lens, fmha), run(rel, pt, lens, fmha)
        assert _err(bc) == (0, 0) and torch.equal(o1, o2)
        bad = pt.clone()
        bad[1, 64:80] = S + torch.arange(page, dtype=torch.int32)
        run(bc, bad, lens, fmha)
        assert _err(bc) == (BOUNDS, SITE_ATTN_SLOT)
        run(bc, pt, [40, stride + 16, 17], fmha)
        assert _err(bc) == (BOUNDS, SITE_ROW)


def test_moe_gather_and_combine_rows(bc):
    T, H, topk = 4, 256, 2
    bigx = torch.randn(T + 4, H, device=DEV).bfloat16()
    xs = torch.empty(8, H, device=DEV, dtype=torch.bfloat16)
    perm = torch.tensor([0, 1, 2, 3, 4, 5, 6, T * topk], dtype=torch.int32, device=DEV)
    bc.moe_gather(xs, bigx[:T], perm, topk)
    assert _err(bc) == (BOUNDS, SITE_PERM)
    assert int(xs[7].float().abs().sum()) == 0  # treated as a padding row
    bigy = torch.randn(T * topk + 4, H, device=DEV).bfloat16()
    out = torch.empty(T, H, device=DEV, dtype=torch.bfloat16)
    w = torch.ones(T, topk, device=DEV)
    inv = torch.arange(T * topk, dtype=torch.int32, device=DEV)
    inv[5] = T * topk
    bc.moe_combine(out, bigy[: T * topk], w, inv, topk)
    assert _err(bc) == (BOUNDS, SITE_INV)


WORKER = r"""
import os, sys
sys.path.insert(0, {root!r})
import torch
from minisgl.core import SamplingParams
from minisgl.llm import LLM
from minisgl._native import cuda
llm = LLM({path!r}, dtype=torch.bfloat16, max_running_req=8, cuda_graph_max_bs=4, num_page_override=512,
          distributed_port={port})
out = llm.generate([[1, 2, 3, 4, 5, 6, 7, 8], list(range(20, 90))], SamplingParams(max_tokens=12, ignore_eos=True))
print("MODULE", type(cuda()._mod).__name__, cuda()._mod.__name__)
print("ERR", tuple(cuda().get_error()))
print("TOKENS", [o["token_ids"] for o in out])
llm.shutdown()
"""


def test_engine_runs_clean_under_bounds_check(tmp_path, free_port):
    """The whole tiny model (prefill, graph-captured decode, sampling) on the bounds-check build:
    no violation recorded, and the same tokens as the release build."""
    from minisgl.models.synthetic import make_checkpoint

    path = make_checkpoint("tiny-qwen3", str(tmp_path / "m"), weights=True)
    outs = {}
    for i, flag in enumerate(("1", "0")):
        script = tmp_path / f"w{flag}.py"
        script.write_text(WORKER.format(root=ROOT, path=path, port=free_port + 7 * i))
        env = dict(os.environ, MINISGL_BOUNDS_CHECK=flag)
        r = subprocess.run([sys.executable, str(script)], env=env, capture_output=True, text=True, timeout=600)
        assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
        lines = {l.split(" ", 1)[0]: l.split(" ", 1)[1] for l in r.stdout.splitlines() if " " in l}
        assert lines["ERR"] == "(0, 0)", r.stdout
        assert lines["MODULE"].endswith("_cuda_bc" if flag == "1" else "_cuda"), lines["MODULE"]
        outs[flag] = lines["TOKENS"]
    assert outs["1"] == outs["0"]
