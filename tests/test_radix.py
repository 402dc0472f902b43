"""Paged KV pool and radix prefix cache (CPU)."""
import pytest

from fak_b200.kv import OutOfPages, PagePool, RadixCache


def test_pool_refcounts():
    p = PagePool(8, reserve=1)
    a = p.alloc(3)
    assert 0 not in a and p.n_free() == 4
    p.retain(a[:1])
    p.release(a)
    assert p.n_free() == 6
    p.release(a[:1])
    assert p.n_free() == 7
    with pytest.raises(OutOfPages):
        p.alloc(8)
    with pytest.raises(RuntimeError):
        p.release(a[:1])


def test_radix_match_insert_split_evict():
    pool = PagePool(64, reserve=1)
    rc = RadixCache(pool, page_size=4)
    t1 = list(range(12))
    pages1 = pool.alloc(3)
    assert rc.insert(t1, pages1) == 12
    pool.release(pages1)  # sequence done: only the tree holds them now
    n, pages = rc.lookup(t1 + [99])
    assert n == 12 and pages == pages1
    pool.release(pages)
    # diverge after 8 tokens -> split
    t2 = list(range(8)) + [50, 51, 52, 53]
    pages2 = pages1[:2] + pool.alloc(1)
    pool.retain(pages1[:2])
    assert rc.insert(t2, pages2) == 4
    pool.release(pages2)
    n, pages = rc.lookup(t2)
    assert n == 12 and pages == pages2
    pool.release(pages)
    n, _ = rc.lookup(list(range(6)))
    assert n == 4  # whole pages only
    pool.release(_)
    free0 = pool.n_free()
    assert rc.evict(2) == 2
    assert pool.n_free() == free0 + 2
    st = rc.stats()
    assert st["hit_tokens"] > 0 and 0 < st["hit_rate"] <= 1


def test_radix_does_not_evict_live_pages():
    pool = PagePool(16, reserve=1)
    rc = RadixCache(pool, page_size=4)
    t = list(range(8))
    pg = pool.alloc(2)
    rc.insert(t, pg)
    # pg still referenced by the sequence -> not evictable
    assert rc.evict(10) == 0
    pool.release(pg)
    assert rc.evict(10) == 2
