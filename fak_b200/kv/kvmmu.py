"""KV memory management unit: a span ledger over a request's attention cache, with verdicts
enforced by evicting K/V.

The context MMU (``agentkernel.ctxmmu``) decides that a tool result may not enter the model's
context.  For text that is about to be sent, that decision rewrites the bytes.  For a result whose
tokens are already in a running request's KV cache, ``KVMMU`` enforces it one layer deeper: the
span the result occupies is evicted from every layer (``Engine.evict_span``: later positions are
renumbered and their keys re-rotated), so the model can no longer attend to it.

The ledger records the token span each appended unit (a prompt chunk, a tool result) occupies;
after an eviction the spans after it are renumbered to match the compacted cache.

``AttentionMass`` accumulates how much attention each cached position receives (an attention
observer of the fp32 reference model, or any per-position signal), and ``KVMMU.evict_coldest``
evicts the least-attended blocks outside a protected sink and recent window.

Reference: kvmmu.Context segments / quarantine / compact / ApplyPlan
(internal/kvmmu/kvmmu.go:51-420), the attention-mass accumulator and EvictColdest
(accumulator.go:42-240, attention.go:49-259).
"""
from __future__ import annotations

import dataclasses

import torch

from ..agentkernel.abi import Verdict, VerdictKind


class AttentionMass:
    """Per-position attention mass: observe(layer, probs [H, Tq, Tctx]) adds the probability each
    key position received, summed over heads and queries (all layers)."""

    def __init__(self):
        self.mass = torch.zeros(0, dtype=torch.float64)

    def observe(self, layer: int, probs: torch.Tensor) -> None:
        m = probs.detach().double().sum(dim=(0, 1)).cpu()
        if m.numel() > self.mass.numel():
            self.mass = torch.cat([self.mass, torch.zeros(m.numel() - self.mass.numel(), dtype=torch.float64)])
        self.mass[: m.numel()] += m

    def drop(self, start: int, end: int) -> None:
        """Keep the ledger aligned with a cache whose positions [start, end) were evicted."""
        self.mass = torch.cat([self.mass[:start], self.mass[end:]])


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

    def evict_coldest(self, mass: torch.Tensor, n_blocks: int, block: int = 16, keep_sink: int = 4,
                      keep_recent: int = 64) -> list[tuple[int, int]]:
        """Evict the ``n_blocks`` blocks of ``block`` positions with the least attention mass, never
        touching the first ``keep_sink`` positions, the last ``keep_recent`` ones or a recorded
        segment; returns the evicted spans (original positions)."""
        n = self.r.n_kv
        lo = -(-keep_sink // block) * block
        hi = n - keep_recent
        cands = []
        for a in range(lo, hi - block + 1, block):
            if any(a < s.end and s.start < a + block for s in self.segments):
                continue
            cands.append((float(mass[a:a + block].sum()), a))
        chosen = sorted(a for _, a in sorted(cands)[:max(0, n_blocks)])
        spans = []
        for a in reversed(chosen):   # highest first: earlier positions do not move
            self.engine.evict_span(self.r, a, a + block)
            spans.append((a, a + block))
        for a, b in spans:           # renumber the ledger per evicted block (highest first, original positions)
            for s in self.segments:
                if s.start >= b:
                    s.start -= block
                    s.end -= block
        return sorted(spans)

    def report(self) -> dict:
        return {"segments": [dataclasses.asdict(s) for s in self.segments],
                "evicted": [dataclasses.asdict(s) for s in self.evicted],
                "evicted_positions": sum(s.length for s in self.evicted)}
