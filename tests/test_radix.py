"""Paged KV pool and radix prefix cache (CPU): the Python specification and the C++ implementation."""
import numpy as np
import pytest

from fak_b200.kv import radix as R
from fak_b200.kv import OutOfPages

IMPLS = [pytest.param((R.PyPagePool, R.PyRadixCache), id="python")]
try:
    from fak_b200 import _cpu
    IMPLS.append(pytest.param((_cpu.PagePool, _cpu.RadixCache), id="native"))
except ImportError:
    pass


@pytest.fixture(params=IMPLS)
def impl(request):
    return request.param


def test_pool_refcounts(impl):
    PagePool, _ = impl
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


def test_radix_match_insert_split_evict(impl):
    PagePool, RadixCache = impl
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


def test_radix_does_not_evict_live_pages(impl):
    PagePool, RadixCache = impl
    pool = PagePool(16, reserve=1)
    rc = RadixCache(pool, page_size=4)
    t = list(range(8))
    pg = pool.alloc(2)
    rc.insert(t, pg)
    # pg still referenced by the sequence -> not evictable
    assert rc.evict(10) == 0
    pool.release(pg)
    assert rc.evict(10) == 2


def test_tp_head_and_ffn_assignment():
    from fak_b200.config import preset
    from fak_b200.models.weights import ffn_assignment, head_assignment, vocab_slice
    cfg = preset("qwen2.5-7b")
    for T in (1, 2, 4, 8):
        qs, kvs = [], []
        for r in range(T):
            q, kv = head_assignment(cfg, r, T)
            qs += q
            kvs.append(kv)
            assert all(h // cfg.gqa_group in kv for h in q)  # a rank owns the KV head of each of its q heads
        assert sorted(qs) == list(range(cfg.n_heads))
        spans = [ffn_assignment(cfg.ffn_dim, r, T, 256) for r in range(T)]
        assert spans[0][0] == 0 and spans[-1][1] == cfg.ffn_dim
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        assert all((b - a) % 256 == 0 for a, b in spans)
        vs = [vocab_slice(cfg.vocab_size, r, T) for r in range(T)]
        assert vs[-1][1] == cfg.vocab_size and sum(b - a for a, b in vs) == cfg.vocab_size
    # TP=8 on 28 q heads / 4 KV heads: groups of 7 split 4 + 3
    assert [len(head_assignment(cfg, r, 8)[0]) for r in range(8)] == [4, 3] * 4


def test_native_radix_matches_python_on_agent_turns():
    """Randomised multi-agent turns: both implementations return the same hits, pages and stats."""
    if len(IMPLS) < 2:
        pytest.skip("native extension not built")
    rng = np.random.default_rng(3)
    sims = []
    for PagePool, RadixCache in ((R.PyPagePool, R.PyRadixCache), (_cpu.PagePool, _cpu.RadixCache)):
        pool = PagePool(600, reserve=1)
        rc = RadixCache(pool, 16)
        r2 = np.random.default_rng(3)
        prefix = r2.integers(0, 1000, 512).tolist()
        hist = [list(prefix) for _ in range(4)]
        log = []
        for turn in range(6):
            for a in range(4):
                hist[a] += r2.integers(0, 1000, int(r2.integers(1, 60))).tolist()
                n, pages = rc.lookup(hist[a], max_tokens=len(hist[a]) - 1)
                need = -(-(len(hist[a]) + 20) // 16) - len(pages)
                if pool.n_free() < need:
                    rc.evict(need - pool.n_free())
                allp = pages + pool.alloc(need)
                hist[a] += r2.integers(0, 1000, 20).tolist()
                rc.insert(hist[a], allp)
                pool.release(allp)
                log.append((n, list(pages), pool.n_free()))
        sims.append((log, rc.stats(), rc.n_cached_pages))
    assert sims[0] == sims[1]


def test_radixbench_workloads():
    from fak_b200.benchmarks import radixbench as RB
    import numpy as np
    for name, fn in RB.WORKLOADS.items():
        reqs = fn(np.random.default_rng(0))
        py = RB.run(reqs, 16, native=False)
        assert 0.5 < py["hit_rate"] < 1.0, (name, py)
        if len(IMPLS) > 1:
            assert RB.run(reqs, 16, native=True) == py


def test_sequences_lists_every_cached_path(impl):
    PagePool, RadixCache = impl
    pool = PagePool(64, reserve=1)
    rc = RadixCache(pool, page_size=4)
    pg = pool.alloc(3)
    rc.insert(list(range(12)), pg)
    pool.release(pg)
    pg2 = pg[:2] + pool.alloc(1)
    pool.retain(pg[:2])
    rc.insert(list(range(8)) + [50, 51, 52, 53], pg2)
    pool.release(pg2)
    seqs = rc.sequences()
    assert [t for t, _ in seqs] == [list(range(12)), list(range(8)) + [50, 51, 52, 53]]
    assert [p for _, p in seqs] == [pg, pg2]
