"""Data-parallel replica routing with prefix residency.

``ReplicaRouter`` fronts several model backends (one engine per GPU or node, or upstream servers)
and sends each request to the replica most likely to hold its prompt prefix in its KV cache: every
replica keeps a residency index -- a page-granular radix tree of the prompts routed to it, the same
structure as the engine's prefix cache -- and a request goes to the replica with the longest
matched prefix; ties go to the replica with the fewest requests in flight, then the fewest routed so
far, then round robin.  The
index is bounded (least-recently-used paths are forgotten) so it tracks what a replica's own cache
can still hold.

``RouterBackend`` exposes the router with the backend interface the gateway uses, so one gateway
can serve a fleet of replicas.

Reference: ReplicaRouter (internal/gateway/replica_router.go), prefix-residency routing of the
native P/D cluster (internal/modelengine/native_pd.go:233-520, kv_fleet_routing.go,
residency_router.go).
"""
from __future__ import annotations

import itertools
import threading

from ..kv.radix import PyPagePool, PyRadixCache


class _Residency:
    """Page-granular record of the prompts a replica has seen (no KV behind it)."""

    def __init__(self, page_size: int, budget_pages: int):
        self.ps = page_size
        self.pool = PyPagePool(budget_pages + 1, reserve=1)
        self.tree = PyRadixCache(self.pool, page_size)

    def match(self, ids: list[int]) -> int:
        return self.tree.match(list(ids))[0]

    def record(self, ids: list[int]) -> None:
        n = len(ids) // self.ps
        if n == 0:
            return
        hit, pages, _ = self.tree.match(list(ids))
        need = n - len(pages)
        if need > self.pool.n_free():
            self.tree.evict(need - self.pool.n_free())
        if need > self.pool.n_free():
            return  # larger than the whole budget: not worth remembering
        self.pool.retain(pages)
        fresh = self.pool.alloc(need)
        self.tree.insert(list(ids), pages + fresh)
        self.pool.release(pages + fresh)


class ReplicaRouter:
    def __init__(self, backends: list, page_size: int = 16, budget_pages: int = 1 << 16):
        if not backends:
            raise ValueError("no replicas")
        self.backends = list(backends)
        self.index = [_Residency(page_size, budget_pages) for _ in backends]
        self.inflight = [0] * len(backends)
        self._rr = itertools.count()
        self._lock = threading.Lock()
        self.routed = [0] * len(backends)

    def choose(self, ids: list[int]) -> int:
        with self._lock:
            scores = [ix.match(ids) for ix in self.index]
            best = max(scores)
            cands = [i for i, s in enumerate(scores) if s == best]
            least = min(self.inflight[i] for i in cands)
            cands = [i for i in cands if self.inflight[i] == least]
            fewest = min(self.routed[i] for i in cands)   # then the replica that served the least
            cands = [i for i in cands if self.routed[i] == fewest]
            pick = cands[next(self._rr) % len(cands)]
            self.index[pick].record(ids)
            self.inflight[pick] += 1
            self.routed[pick] += 1
            return pick

    def done(self, i: int) -> None:
        with self._lock:
            self.inflight[i] -= 1

    def stats(self) -> dict:
        return {"replicas": len(self.backends), "routed": list(self.routed), "inflight": list(self.inflight)}


class RouterBackend:
    """Backend interface over a ReplicaRouter (generate streams token ids of the chosen replica)."""

    def __init__(self, router: ReplicaRouter, tokenizer=None, name: str = "fak-b200-fleet"):
        self.router = router
        self.tok = tokenizer if tokenizer is not None else getattr(router.backends[0], "tok", None)
        self.name = name

    def generate(self, prompt_ids: list[int], max_tokens: int, sampling, stop_ids=()):
        i = self.router.choose(list(prompt_ids))
        try:
            yield from self.router.backends[i].generate(prompt_ids, max_tokens, sampling, stop_ids)
        finally:
            self.router.done(i)
