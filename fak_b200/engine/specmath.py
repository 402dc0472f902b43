"""Expected yield of speculative decoding.

With K drafted tokens per verify step and a per-token acceptance probability a (independent),
the number of tokens a verify step emits (accepted drafts plus the target's own token) is
E(K, a) = (1 - a^(K+1)) / (1 - a), which tends to K + 1 as a -> 1 and to 1 as a -> 0.  With a draft
step costing c (relative to one target step, draft = c per drafted token) and a verify step costing
v (relative to one plain decode step), the speed-up over plain decoding is E / (K c + v).
``best_k`` picks the K with the largest speed-up.

Reference: the acceptance arithmetic of internal/polymodel and cmd/polymodelbench (spec-decode
E(K, a)); the acceptance meter of internal/spec/metrics.go:34-110.
"""
from __future__ import annotations

import dataclasses


def expected_tokens(k: int, a: float) -> float:
    if k < 0 or not 0.0 <= a <= 1.0:
        raise ValueError("k >= 0 and 0 <= a <= 1")
    if a == 1.0:
        return float(k + 1)
    return (1.0 - a ** (k + 1)) / (1.0 - a)


def speedup(k: int, a: float, draft_cost: float, verify_cost: float = 1.0) -> float:
    return expected_tokens(k, a) / (k * draft_cost + verify_cost)


def best_k(a: float, draft_cost: float, verify_cost: float = 1.0, k_max: int = 16) -> tuple[int, float]:
    return max(((k, speedup(k, a, draft_cost, verify_cost)) for k in range(k_max + 1)), key=lambda t: t[1])


def acceptance_from_stats(drafted: int, accepted: int) -> float:
    """Per-token acceptance estimate from engine counters (accepted drafts / drafted tokens)."""
    return accepted / drafted if drafted else 0.0


@dataclasses.dataclass
class AcceptanceMeter:
    """Running acceptance over verify steps (drafted / accepted per step)."""
    drafted: int = 0
    accepted: int = 0
    steps: int = 0

    def observe(self, drafted: int, accepted: int) -> None:
        if not 0 <= accepted <= drafted:
            raise ValueError("0 <= accepted <= drafted")
        self.drafted += drafted
        self.accepted += accepted
        self.steps += 1

    @property
    def rate(self) -> float:
        return acceptance_from_stats(self.drafted, self.accepted)

    @property
    def tokens_per_step(self) -> float:
        return (self.accepted + self.steps) / self.steps if self.steps else 0.0
