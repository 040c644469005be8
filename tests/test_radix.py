import numpy as np
import pytest

from minisgl._native import host
from minisgl.kvcache import create_prefix_cache


def a(*x):
    return np.array(x, dtype=np.int32)


def test_compare_key():
    assert host().compare_key(a(1, 2, 3, 4), a(1, 2, 9)) == 2
    assert host().compare_key(a(1, 2), a(1, 2, 3)) == 2


def test_insert_match_split_page1():
    t = host().RadixTree(1)
    pre, h = t.insert(a(1, 2, 3, 4), a(10, 11, 12, 13))
    assert pre == 0 and t.evictable_size == 4
    h2, n = t.match(a(1, 2, 5))
    assert n == 2 and list(t.indices(h2)) == [10, 11]
    # the split created a node for [1,2]; sizes unchanged
    assert t.evictable_size == 4 and t.num_nodes == 3
    pre, h3 = t.insert(a(1, 2, 7, 8), a(20, 21, 22, 23))
    assert pre == 2 and t.evictable_size == 6
    assert list(t.indices(h3)) == [10, 11, 22, 23]
    t.check_integrity()


def test_page_aligned_match():
    t = host().RadixTree(4)
    t.insert(a(*range(12)), a(*range(100, 112)))
    h, n = t.match(a(0, 1, 2, 3, 4, 5, 99, 7, 8))
    assert n == 4  # match rounds down to a page boundary
    assert list(t.indices(h)) == [100, 101, 102, 103]
    pre, _ = t.insert(a(0, 1, 2), a(1, 2, 3))  # shorter than a page: nothing inserted
    assert pre == 0
    t.check_integrity()


def test_lock_evict_lru():
    t = host().RadixTree(1)
    _, h1 = t.insert(a(1, 2, 3), a(1, 2, 3))
    _, h2 = t.insert(a(5, 6), a(5, 6))
    t.lock(h1)
    assert t.protected_size == 3 and t.evictable_size == 2
    with pytest.raises(RuntimeError):
        t.evict(3)
    ev = t.evict(1)
    assert sorted(ev.tolist()) == [5, 6]
    t.unlock(h1)
    with pytest.raises(RuntimeError):
        t.lock(h2)  # h2's node was evicted: handle is stale
    assert sorted(t.evict(3).tolist()) == [1, 2, 3]
    assert t.evictable_size == 0 and t.num_nodes == 1
    t.check_integrity()


def test_evict_cascades_to_parent_lru_order():
    t = host().RadixTree(1)
    t.insert(a(1, 2, 3), a(1, 2, 3))
    t.insert(a(1, 2, 4), a(1, 2, 4))  # splits: [1,2] -> {[3],[4]}
    t.match(a(1, 2, 4))  # touch the [4] branch
    ev = t.evict(1)
    assert ev.tolist() == [3]  # least recently used leaf first
    ev = t.evict(3)
    assert sorted(ev.tolist()) == [1, 2, 4]
    t.check_integrity()


def test_prefix_cache_wrapper():
    c = create_prefix_cache("radix", page_size=2)
    r = c.insert_prefix(np.arange(5, dtype=np.int32), np.arange(50, 55, dtype=np.int32))
    assert r.cached_len == 0 and r.handle.cached_len == 4
    m = c.match_prefix(np.arange(5, dtype=np.int32)).cuda_handle
    assert m.cached_len == 4 and m.get_matched_indices().tolist() == [50, 51, 52, 53]
    c.lock_handle(m)
    assert c.size_info.protected_size == 4
    c.lock_handle(m, unlock=True)
    assert c.size_info.evictable_size == 4
    c.check_integrity()


def test_random_ops_integrity():
    rng = np.random.default_rng(0)
    t = host().RadixTree(2)
    handles = []
    for _ in range(300):
        op = rng.integers(0, 4)
        if op == 0:
            n = int(rng.integers(1, 20))
            ids = rng.integers(0, 4, n).astype(np.int32)
            _, h = t.insert(ids, np.arange(n, dtype=np.int32))
            t.lock(h)
            handles.append(h)
        elif op == 1 and handles:
            t.unlock(handles.pop(int(rng.integers(0, len(handles)))))
        elif op == 2:
            t.match(rng.integers(0, 4, int(rng.integers(1, 20))).astype(np.int32))
        elif op == 3 and t.evictable_size > 0:
            t.evict(int(rng.integers(1, t.evictable_size + 1)))
        t.check_integrity()
