"""Page allocator + prefix cache (CPU): page-aligned allocation after radix eviction, no page owned
twice, the decode fast path of ``allocate_paged`` equal to the general path, and the
free + cached == total invariant through random admit / extend / cache / finish cycles
(the reference's suite: tests/core/test_cache_allocate.py:58-199)."""

import numpy as np
import pytest
import torch

from minisgl.core import Req, SamplingParams
from minisgl.scheduler.cache import CacheManager


def admit(cm, ids, row, uid, out_len=8):
    """What the prefill adder does for one request: match, lock, build the Req."""
    m = cm.match_req(torch.tensor(ids, dtype=torch.int32))
    h = m.cuda_handle
    cm.lock(h)
    r = Req(torch.tensor(ids, dtype=torch.int32), row, h.cached_len, out_len, uid, SamplingParams(), h)
    r.slots = np.asarray(h.get_matched_indices(), dtype=np.int32)
    r.pending_prefix = h.cached_len
    return r


def live_pages(reqs, ps):
    """Pages each request wrote itself (beyond its matched prefix)."""
    out = []
    for r in reqs:
        own = r.slots[r.cache_handle.cached_len : r.cached_len]
        out.extend(np.unique(own // ps).tolist())
    return out


@pytest.mark.parametrize("ps", [1, 4, 8])
def test_random_cycles_keep_integrity(ps):
    rng = np.random.default_rng(ps)
    cm = CacheManager(num_pages=64, page_size=ps, cache_type="radix")
    roots = [rng.integers(0, 50, 48).tolist() for _ in range(3)]
    live, uid = [], 0
    for step in range(300):
        act = rng.random()
        if act < 0.35 and len(live) < 6:
            root = roots[int(rng.integers(0, 3))]
            ids = root[: int(rng.integers(1, 48))] + rng.integers(0, 50, int(rng.integers(1, 12))).tolist()
            need = len(ids) + 8 + ps
            if need > cm.available_size - sum(r.max_device_len - r.cached_len + ps for r in live):
                continue
            r = admit(cm, ids, uid % 8, uid)
            uid += 1
            rows, pos, slots = cm.allocate_paged([r])
            r.complete_one()
            # page-table writes cover the matched prefix and the new pages, page-aligned
            assert np.all(slots[pos % ps == 0] % ps == 0)
            assert np.array_equal(slots, r.slots[pos])
            cm.cache_req(r, finished=False)
            live.append(r)
        elif act < 0.8 and live:
            batch = [r for r in live if r.device_len < r.max_device_len]
            if batch:
                cm.allocate_paged(batch)
                for r in batch:
                    r.complete_one()
                    r.append_host(int(rng.integers(0, 50)))
        elif live:
            r = live.pop(int(rng.integers(0, len(live))))
            cm.cache_req(r, finished=True)
        pages = live_pages(live, ps)
        assert len(pages) == len(set(pages)), f"page owned twice at step {step}"
        cm.check_integrity() if not live else cm.prefix_cache.check_integrity()
    for r in live:
        cm.cache_req(r, finished=True)
    cm.check_integrity()
    assert cm.available_size == 64 * ps


@pytest.mark.parametrize("ps", [4, 16])
def test_decode_fast_path_matches_general_allocation(ps):
    """A decode step needs a page only when the token starts one; those pages come first-fit
    from the free list in batch order, as the general path would give them."""
    cm = CacheManager(num_pages=32, page_size=ps, cache_type="radix")
    reqs = []
    for i, n in enumerate([ps, ps + 1, 2 * ps - 1, 3 * ps]):
        r = Req(torch.arange(n, dtype=torch.int32) + 100 * i, i, 0, 4, i, SamplingParams(),
                cm.match_req(torch.arange(n, dtype=torch.int32) + 100 * i).cuda_handle)
        r.slots = np.empty(0, np.int32)
        reqs.append(r)
    cm.allocate_paged(reqs)
    for r in reqs:
        r.complete_one()
    free_before = cm.free_pages.copy()
    rows, pos, slots = cm.allocate_paged(reqs)  # one token each
    starts = [r for r in reqs if r.cached_len % ps == 0]
    assert len(rows) == len(starts) * ps
    assert slots[::ps].tolist() == free_before[: len(starts)].tolist()
    for r in reqs:
        first = r.slots[r.cached_len]
        assert first == r.slots[r.cached_len - 1] + 1 or r.cached_len % ps == 0


def test_eviction_refills_free_list_page_aligned():
    ps = 8
    cm = CacheManager(num_pages=8, page_size=ps, cache_type="radix")
    done = []
    for i in range(4):  # fill the cache with 4 finished 2-page prompts
        r = admit(cm, (np.arange(16) + 100 * i).tolist(), i, i)
        cm.allocate_paged([r])
        r.complete_one()
        cm.cache_req(r, finished=True)
        done.append(r)
    assert len(cm.free_pages) == 0 and cm.available_size == 64
    r = admit(cm, (np.arange(40) + 999).tolist(), 0, 9)
    rows, pos, slots = cm.allocate_paged([r])  # needs 5 pages: evicts 5 of the cached ones
    assert len(slots) == 40 and len(set((slots // ps).tolist())) == 5
    assert np.all(slots.reshape(5, ps) - slots.reshape(5, ps)[:, :1] == np.arange(ps))
    r.complete_one()
    cm.cache_req(r, finished=True)
    cm.check_integrity()
