"""Host-side planning of the persistent decode attention kernel (CPU): the work list must cover
every 64-key block of every request exactly once, in longest-first order, with per-request chunk
numbering and partial-slot offsets the kernel's combine relies on."""

import numpy as np
import pytest

from minisgl.attention.paged import decode_work_list


@pytest.mark.parametrize("num_ctas,max_entries", [(148, None), (3, None), (148, 40), (1, 7)])
@pytest.mark.parametrize("seed", [0, 1])
def test_work_list_covers_every_block_once(num_ctas, max_entries, seed):
    rng = np.random.default_rng(seed)
    lens = rng.integers(1, 9000, 37)
    lens[3] = 64 * 128 * 9  # a request that needs the per-request chunk cap (<= 128 chunks)
    w, n = decode_work_list(lens, kv_heads=8, num_ctas=num_ctas, max_entries=max_entries)
    e = w.reshape(n, 8)
    nblk = (lens + 63) // 64
    seen = [np.zeros(k, np.int32) for k in nblk]
    for b, blk0, blk1, j, nch, slot0, _, _ in e:
        assert 0 <= blk0 < blk1 <= nblk[b]
        seen[b][blk0:blk1] += 1
        assert 0 <= j < nch <= 128
    assert all((s == 1).all() for s in seen)
    # longest first
    length = e[:, 2] - e[:, 1]
    assert (np.diff(length) <= 0).all()
    # chunk indices 0..nch-1 once per request; partial slots are disjoint ranges in request order
    for b in range(len(lens)):
        rows = e[e[:, 0] == b]
        nch = rows[0, 4]
        assert sorted(rows[:, 3].tolist()) == list(range(nch))
        assert (rows[:, 4] == nch).all() and (rows[:, 5] == rows[0, 5]).all()
    slot0 = [int(e[e[:, 0] == b][0, 5]) for b in range(len(lens))]
    nchs = [int(e[e[:, 0] == b][0, 4]) for b in range(len(lens))]
    assert slot0 == [0] + np.cumsum(nchs[:-1]).tolist()
    if max_entries is not None:
        # the chunk length grows until the entries fit; every request needs at least one entry
        assert n <= max(max_entries, len(lens)), (n, max_entries)


def test_work_list_empty_and_single():
    w, n = decode_work_list(np.zeros(0, np.int64), 8, 148)
    assert n == 0 and w.size == 0
    w, n = decode_work_list(np.array([1]), 1, 148)
    assert n == 1 and w.reshape(1, 8)[0, :5].tolist() == [0, 0, 1, 0, 1]
