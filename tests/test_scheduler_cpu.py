"""Scheduler, cache manager and batch plan under a fake model (CPU, no GPU).

The real engine runs (page table, batch plan upload, out_loc, last-token rows, greedy sampler) with
the model replaced by a rule whose next token is a function of (last token, position):

    next = (7 * token + 3 * position + 1) mod V

so every request's output is known from its prompt alone, whatever the scheduler does with it:
chunked prefill, prefix-cache hits, queueing behind a small running set or a tight KV pool, EOS.
The fake model also checks, on every forward, that the KV slots it is about to write belong to no
other live request (shared prefix slots are only ever read).
"""

import numpy as np
import pytest
import torch

from minisgl.core import SamplingParams, get_global_ctx
from minisgl.models.synthetic import make_checkpoint

V = 1000


def rule(tok: int, pos: int) -> int:
    return (7 * tok + 3 * pos + 1) % V


def expected(prompt, n, eos=None):
    out, tok, pos = [], prompt[-1], len(prompt) - 1
    for _ in range(n):
        tok = rule(tok, pos)
        pos += 1
        if tok == eos:
            break
        out.append(tok)
    return out


class FakeModel:
    """Stands in for the network. Besides producing the rule's token it keeps a mirror of the KV
    pool (slot -> (token, position) written there) and checks that every position a request would
    attend to maps to a slot holding exactly that request's (token, position)."""

    def __init__(self, engine):
        self.engine = engine
        self.forwards = 0
        self.prefill_tokens = 0  # prompt tokens actually computed (prefix-cache hits excluded)
        self.kv = {}

    def _check_kv(self, batch):
        # the tokens this forward writes come from the device input (under overlap scheduling the
        # host copy of a decode request still lacks the token sampled by the previous step)
        toks = batch.input_ids.tolist()
        k = 0
        for r in batch.padded_reqs:
            for p in range(r.cached_len, r.device_len):
                if r in batch.reqs:
                    self.kv[int(r.slots[p])] = (toks[k], p)
                k += 1
        for r in batch.reqs:
            ids = r.input_ids.tolist()
            n = min(len(ids), r.device_len)
            got = [self.kv.get(int(s)) for s in r.slots[:n]]
            bad = [p for p in range(n) if got[p] != (ids[p], p)]
            assert not bad, f"req {r.uid}: positions {bad[:8]} read KV written for another token"

    def forward(self):
        ctx = get_global_ctx()
        b = ctx.batch
        self.forwards += 1
        if b.is_prefill:
            self.prefill_tokens += sum(r.device_len - r.cached_len for r in b.reqs)
        self._check_kv(b)
        # out_loc must be the page-table slots of the extend tokens
        want = np.concatenate([r.slots[r.cached_len : r.device_len] for r in b.padded_reqs])
        assert b.out_loc.tolist() == want.tolist()
        idx = b.attn_metadata.get_last_indices(b.size)
        tok = b.input_ids[idx].long()
        pos = b.positions[idx].long()
        nxt = (7 * tok + 3 * pos + 1) % V
        logits = torch.zeros(b.size, V)
        logits[torch.arange(b.size), nxt] = 1.0
        return logits


@pytest.fixture(scope="module")
def tiny_path(tmp_path_factory):
    return make_checkpoint("tiny-qwen3", str(tmp_path_factory.mktemp("m")))


def make_llm(path, port, **kw):
    from minisgl.llm import LLM

    kw.setdefault("max_running_req", 8)
    llm = LLM(path, dtype=torch.float32, device="cpu", use_dummy_weight=True, distributed_port=port, **kw)
    llm.engine.model = FakeModel(llm.engine)
    return llm


def prompts_with_shared_prefixes(seed, n, lo=5, hi=90):
    g = np.random.default_rng(seed)
    roots = [g.integers(0, V, 40).tolist() for _ in range(3)]
    out = []
    for i in range(n):
        if i % 3 == 0:
            out.append(g.integers(0, V, int(g.integers(lo, hi))).tolist())
        else:  # a shared prefix of 8..40 tokens plus a private tail
            root = roots[i % 3][: int(g.integers(8, 41))]
            out.append(root + g.integers(0, V, int(g.integers(1, 30))).tolist())
    return out


@pytest.mark.parametrize(
    "page,cache,budget,running,pages",
    [
        (1, "radix", 16384, 8, None),
        (4, "radix", 32, 4, None),  # chunked prefill: prompts longer than the per-step budget
        (16, "radix", 64, 3, 24),  # tight pool: requests queue for pages
        (8, "naive", 48, 8, None),
        (64, "radix", 16384, 16, None),
    ],
)
def test_fake_model_outputs(tiny_path, free_port, page, cache, budget, running, pages):
    llm = make_llm(tiny_path, free_port, page_size=page, cache_type=cache, max_extend_tokens=budget,
                   max_running_req=running, num_page_override=pages)
    try:
        prompts = prompts_with_shared_prefixes(page, 18)
        lens = [3 + (i * 5) % 23 for i in range(len(prompts))]
        sps = [SamplingParams(max_tokens=n, ignore_eos=True) for n in lens]
        computed = []
        for rep in range(2):  # the second pass hits the prefix cache left by the first
            fm = llm.engine.model
            before = fm.prefill_tokens
            outs = llm.generate(prompts, sps)
            for p, n, o in zip(prompts, lens, outs):
                assert o["token_ids"] == expected(p, n), (rep, p)
            llm.cache_manager.check_integrity()
            computed.append(fm.prefill_tokens - before)
        total = sum(len(p) for p in prompts)
        assert computed[0] <= total
        if cache == "naive":
            assert computed == [total, total]
        elif pages is None:
            # the first pass left every prompt cached (evictable, nothing evicted): the second pass
            # reuses each prompt's whole pages short of its last token and computes the rest
            assert computed[1] == sum(len(p) - (len(p) - 1) // page * page for p in prompts), computed
        else:
            assert computed[1] <= computed[0]
        cm = llm.cache_manager
        assert cm.available_size == cm.num_pages * cm.page_size  # every page free or evictable
        assert not llm.decode_manager.running and not llm.prefill_manager.pending_list
    finally:
        llm.shutdown()


def test_eos_stops_and_is_not_returned(tiny_path, free_port):
    llm = make_llm(tiny_path, free_port)
    try:
        eos = llm.eos_token_id
        assert eos is not None and eos < V
        # prompts whose continuation reaches EOS at a known step: solve rule(tok, pos) == eos
        prompts, want = [], []
        for L in (6, 11, 17):
            pos = L - 1
            tok = next(t for t in range(V) if rule(t, pos) == eos)
            prompts.append([5] * (L - 1) + [tok])
            want.append([])
        prompts.append([1, 2, 3])
        want.append(expected([1, 2, 3], 12, eos))
        outs = llm.generate(prompts, SamplingParams(max_tokens=12))
        assert [o["token_ids"] for o in outs] == want
        ign = llm.generate(prompts[:1], SamplingParams(max_tokens=4, ignore_eos=True))
        assert ign[0]["token_ids"] == expected(prompts[0], 4) and ign[0]["token_ids"][0] == eos
        llm.cache_manager.check_integrity()
    finally:
        llm.shutdown()


def test_max_tokens_clamped_to_context(tiny_path, free_port):
    llm = make_llm(tiny_path, free_port, max_seq_len_override=64)
    try:
        p = list(range(1, 51))
        out = llm.generate([p], SamplingParams(max_tokens=100, ignore_eos=True))[0]["token_ids"]
        assert out == expected(p, 14)  # 64 - 50 tokens of room
    finally:
        llm.shutdown()


def test_concurrent_requests_with_one_uncached_prefix(tiny_path, free_port):
    """Requests that share a prefix nobody has cached yet are prefilled side by side, each into its
    own pages. When the first inserts the prefix, the others' copies become redundant and go back
    to the free list; the requests still decoding must then read the cached copy, not their freed
    pages, which new requests are about to overwrite."""
    llm = make_llm(tiny_path, free_port, page_size=4, max_running_req=6, num_page_override=64)
    try:
        g = np.random.default_rng(1)
        root = g.integers(0, V, 32).tolist()
        prompts = [root + g.integers(0, V, 6).tolist() for _ in range(6)]
        prompts += [g.integers(0, V, 30).tolist() for _ in range(12)]
        lens = [40] * 6 + [10] * 12
        outs = llm.generate(prompts, [SamplingParams(max_tokens=n, ignore_eos=True) for n in lens])
        for p, n, o in zip(prompts, lens, outs):
            assert o["token_ids"] == expected(p, n)
        llm.cache_manager.check_integrity()
    finally:
        llm.shutdown()


def run_overlapped(llm):
    """The overlap loop (schedule and launch batch N+1 before processing batch N's results), which
    the engine uses on CUDA, driven on the CPU engine."""

    def loop():
        data = None
        while True:
            data = llm.overlap_loop(data)

    llm.run_forever = loop


@pytest.mark.parametrize("page", [1, 16])
def test_overlap_loop_with_eos_stops(tiny_path, free_port, page):
    """Under overlap scheduling a request that stops on EOS is already part of the next batch;
    that surplus step's token must not reach the output, and the request's pages are freed once."""
    llm = make_llm(tiny_path, free_port, page_size=page, max_running_req=6, max_extend_tokens=64)
    run_overlapped(llm)
    try:
        eos = llm.eos_token_id
        prompts, want = [], []
        g = np.random.default_rng(3)
        for i in range(10):
            L = int(g.integers(4, 40))
            if i % 2 == 0:  # reaches EOS after i // 2 + 1 generated tokens
                prompt = g.integers(0, V, L).tolist()
                k = i // 2 + 1
                # choose the last prompt token so that the k-th generated token is EOS
                for t in range(V):
                    prompt[-1] = t
                    seq = expected(prompt, k)
                    if seq[-1] == eos and eos not in seq[:-1]:
                        break
                prompts.append(prompt)
                want.append(expected(prompt, 20, eos))
                assert len(want[-1]) == k - 1
            else:
                prompts.append(g.integers(0, V, L).tolist())
                want.append(expected(prompts[-1], 20, eos))
        for _ in range(2):
            outs = llm.generate(prompts, SamplingParams(max_tokens=20))
            assert [o["token_ids"] for o in outs] == want
            llm.cache_manager.check_integrity()
        cm = llm.cache_manager
        assert cm.available_size == cm.num_pages * cm.page_size
    finally:
        llm.shutdown()


def test_overlap_loop_outputs(tiny_path, free_port):
    llm = make_llm(tiny_path, free_port, page_size=4, max_extend_tokens=32, max_running_req=4, num_page_override=40)
    run_overlapped(llm)
    try:
        prompts = prompts_with_shared_prefixes(7, 14)
        lens = [3 + (i * 5) % 23 for i in range(len(prompts))]
        outs = llm.generate(prompts, [SamplingParams(max_tokens=n, ignore_eos=True) for n in lens])
        for p, n, o in zip(prompts, lens, outs):
            assert o["token_ids"] == expected(p, n)
        llm.cache_manager.check_integrity()
    finally:
        llm.shutdown()


@pytest.mark.parametrize("overlap", [False, True])
def test_aborts_free_everything_once(tiny_path, free_port, overlap):
    """Requests aborted while pending, mid-chunked-prefill and mid-decode: the others still produce
    their exact outputs, an aborted request's pages and table row are released exactly once
    (also when a batch holding it was already in flight), and the pool ends whole."""
    from minisgl.message import AbortBackendMsg

    llm = make_llm(tiny_path, free_port, page_size=4, max_extend_tokens=24, max_running_req=4, num_page_override=60)
    if overlap:
        run_overlapped(llm)
    g = np.random.default_rng(11)
    prompts = [g.integers(0, V, int(g.integers(10, 60))).tolist() for _ in range(12)]
    # uid -> receive call at which its abort arrives: spread so that aborts land while the
    # request is pending, mid-chunk, just launched (prefill in flight) and decoding
    plan = {0: 2, 1: 3, 3: 4, 5: 1, 6: 5, 7: 6, 9: 9, 11: 12}
    orig = llm.receive_msg
    calls = [0]

    def receive(blocking=False):
        msgs = list(orig(blocking=blocking))
        calls[0] += 1
        msgs += [AbortBackendMsg(uid=u) for u, c in plan.items() if c == calls[0]]
        return msgs

    llm.receive_msg = receive  # (TableManager.free raises on a row freed twice)
    try:
        outs = llm.generate(prompts, SamplingParams(max_tokens=15, ignore_eos=True))
        for i, (p, o) in enumerate(zip(prompts, outs)):
            want = expected(p, 15)
            if i in plan:
                assert o["token_ids"] == want[: len(o["token_ids"])]  # a prefix of the full output
            else:
                assert o["token_ids"] == want, i
        llm.cache_manager.check_integrity()
        cm = llm.cache_manager
        assert cm.available_size == cm.num_pages * cm.page_size
        assert llm.table_manager.available_size == 4
        assert not llm.decode_manager.running and not llm.prefill_manager.pending_list
    finally:
        llm.shutdown()


def test_rejected_requests_finish_empty(tiny_path, free_port):
    """An empty prompt, a prompt at the context limit and max_tokens = 0 are answered at once with
    no tokens (instead of being dropped, which left their clients waiting); the rest run."""
    llm = make_llm(tiny_path, free_port, max_seq_len_override=64)
    try:
        prompts = [[], list(range(1, 65)), [5, 6, 7], [8, 9]]
        sps = [SamplingParams(max_tokens=4, ignore_eos=True)] * 2 + [
            SamplingParams(max_tokens=0, ignore_eos=True), SamplingParams(max_tokens=4, ignore_eos=True)]
        outs = [o["token_ids"] for o in llm.generate(prompts, sps)]
        assert outs == [[], [], [], expected([8, 9], 4)]
        llm.cache_manager.check_integrity()
    finally:
        llm.shutdown()
