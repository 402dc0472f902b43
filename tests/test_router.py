"""Data-parallel replica routing by prefix residency (CPU, fake replicas)."""
from fak_b200.serve.router import ReplicaRouter, RouterBackend


class Echo:
    def __init__(self, name):
        self.name, self.seen = name, []

    def generate(self, ids, max_tokens, sampling, stop_ids=()):
        self.seen.append(list(ids))
        yield from range(max_tokens)


def test_agents_stick_to_the_replica_holding_their_prefix():
    reps = [Echo(i) for i in range(3)]
    r = ReplicaRouter(reps, page_size=4)
    be = RouterBackend(r)
    sys_a, sys_b = list(range(100, 164)), list(range(500, 564))
    hist = {a: (sys_a if a < 3 else sys_b) + [a] * 8 for a in range(6)}
    for turn in range(4):
        for a in range(6):
            hist[a] = hist[a] + [1000 + turn * 10 + a] * 8
            assert list(be.generate(hist[a], 2, None)) == [0, 1]
    owners = {}
    for i, rep in enumerate(reps):
        for ids in rep.seen:
            owners.setdefault(ids[0], set()).add(i)
    # each system prefix lives on one replica after the first request of its family
    assert all(len(s) == 1 for s in owners.values()), owners
    assert owners[100] != owners[500]
    assert r.stats()["inflight"] == [0, 0, 0] and sum(r.stats()["routed"]) == 24


def test_ties_balance_by_load_then_round_robin():
    reps = [Echo(i) for i in range(2)]
    r = ReplicaRouter(reps, page_size=4)
    a = r.choose([1, 2, 3, 4, 5, 6, 7, 8])
    b = r.choose([9, 10, 11, 12, 13, 14, 15, 16])   # no shared prefix: the idle replica
    assert a != b
    r.done(a)
    r.done(b)


def test_residency_is_bounded():
    r = ReplicaRouter([Echo(0)], page_size=4, budget_pages=8)
    for k in range(20):
        r.choose([k] * 16)
        r.done(0)
    assert r.index[0].pool.n_free() >= 0 and r.index[0].match([19] * 16) == 16
