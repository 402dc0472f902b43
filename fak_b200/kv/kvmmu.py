"""KV memory management unit: a span ledger over a request's attention cache, with verdicts
enforced by evicting K/V.

The context MMU (``agentkernel.ctxmmu``) decides that a tool result may not enter the model's
context.  For text that is about to be sent, that decision rewrites the bytes.  For a result whose
tokens are already in a running request's KV cache, ``KVMMU`` enforces it one layer deeper: the
span the result occupies is evicted from every layer (``Engine.evict_span``: later positions are
renumbered and their keys re-rotated), so the model can no longer attend to it.

The ledger records the token span each appended unit (a prompt chunk, a tool result) occupies;
after an eviction the spans after it are renumbered to match the compacted cache.

Reference: kvmmu.Context segments / quarantine / compact / ApplyPlan
(internal/kvmmu/kvmmu.go:51-420).
"""
from __future__ import annotations

import dataclasses

from ..agentkernel.abi import Verdict, VerdictKind


@dataclasses.dataclass
class Segment:
    id: str
    start: int
    end: int
    tool: str = ""

    @property
    def length(self) -> int:
        return self.end - self.start


class KVMMU:
    """Span ledger for one decoding request of ``engine`` (``Engine`` or anything with
    ``evict_span(request, start, end)``)."""

    EVICTING = (VerdictKind.QUARANTINE, VerdictKind.DENY)

    def __init__(self, engine, request):
        self.engine = engine
        self.r = request
        self.segments: list[Segment] = []
        self.evicted: list[Segment] = []

    def record(self, seg_id: str, start: int, end: int, tool: str = "") -> Segment:
        if not 0 <= start < end:
            raise ValueError(f"segment {seg_id}: empty or negative span [{start}, {end})")
        if any(s.id == seg_id for s in self.segments):
            raise ValueError(f"segment {seg_id} already recorded")
        for s in self.segments:
            if start < s.end and s.start < end:
                raise ValueError(f"segment {seg_id} [{start}, {end}) overlaps {s.id} [{s.start}, {s.end})")
        seg = Segment(seg_id, start, end, tool)
        self.segments.append(seg)
        self.segments.sort(key=lambda s: s.start)
        return seg

    def append(self, seg_id: str, n_tokens: int, tool: str = "") -> Segment:
        """Record the last ``n_tokens`` positions of the request's cache as one segment."""
        end = self.r.n_kv
        return self.record(seg_id, end - n_tokens, end, tool)

    def quarantine(self, seg_id: str) -> int:
        """Evict a segment's K/V; returns the positions removed."""
        seg = next((s for s in self.segments if s.id == seg_id), None)
        if seg is None:
            raise KeyError(seg_id)
        n = self.engine.evict_span(self.r, seg.start, seg.end)
        self.segments.remove(seg)
        self.evicted.append(seg)
        for s in self.segments:
            if s.start >= seg.end:
                s.start -= n
                s.end -= n
        return n

    def apply(self, verdict: Verdict, seg_id: str) -> int:
        """Enforce a context-admission verdict on a recorded segment (quarantine / deny evict it)."""
        return self.quarantine(seg_id) if verdict.kind in self.EVICTING else 0

    def report(self) -> dict:
        return {"segments": [dataclasses.asdict(s) for s in self.segments],
                "evicted": [dataclasses.asdict(s) for s in self.evicted],
                "evicted_positions": sum(s.length for s in self.evicted)}
