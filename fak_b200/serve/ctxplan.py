"""Context planner: each turn's prompt is a planned view over the full conversation, kept inside a
token budget, instead of the whole transcript (which outgrows the window) or a lossy summary.

The conversation is a list of cells (messages).  A ``Layout`` splits it into areas:

* base    -- pinned structural material: system / developer messages (always resident);
* current -- the newest ``current_n`` messages (always resident, exact);
* recent  -- the ``recent_n`` messages before them (resident while they fit, exact);
* deep    -- everything older: resident only when its benefit earns its tokens.

Each deep cell gets a benefit from three signals combined with ``Weights``: relevance to the
forecast (the current turn's text: smoothed inverse-document-frequency weighted term overlap),
recency (exponential decay with age) and durability (system-like content, tool results that were
referenced again later).  ``plan`` solves the budgeted 0/1 knapsack over the deep cells (exact
dynamic programming over token costs bucketed to ``granule`` tokens) after the pinned areas are
charged; cells that do not make it are replaced by one-line pointers naming the cell and its size
(a later turn can page it back in by id), in original order so the view stays a readable
transcript.  ``Plan.explain`` lists every cell with its area, tokens, benefit and decision.

Reference: internal/ctxplan (doc.go: Layout areas base / current / recent / deep, Forecast weights,
Optimize as a budgeted 0/1 knapsack, Plan.Explain, pointer precision for elided spans).
"""
from __future__ import annotations

import dataclasses
import math
import re
from typing import Callable

_WORD = re.compile(r"[A-Za-z0-9_./-]{2,}")


def _terms(text: str) -> list[str]:
    return [w.lower() for w in _WORD.findall(text or "")]


def _text(msg: dict) -> str:
    c = msg.get("content")
    if isinstance(c, list):   # OpenAI content parts
        return " ".join(p.get("text", "") for p in c if isinstance(p, dict))
    return c if isinstance(c, str) else ("" if c is None else str(c))


@dataclasses.dataclass
class Weights:
    relevance: float = 1.0
    recency: float = 0.5
    durability: float = 0.5
    half_life: float = 8.0     # messages


@dataclasses.dataclass
class Layout:
    current_n: int = 2
    recent_n: int = 6
    granule: int = 16          # tokens per knapsack bucket


@dataclasses.dataclass
class CellPlan:
    index: int
    area: str
    tokens: int
    benefit: float
    resident: bool


@dataclasses.dataclass
class Plan:
    cells: list[CellPlan]
    budget: int
    resident_tokens: int
    messages: list[dict]

    def explain(self) -> list[dict]:
        return [dataclasses.asdict(c) for c in self.cells]


class ContextPlanner:
    def __init__(self, budget_tokens: int, count_tokens: Callable[[str], int] | None = None,
                 layout: Layout | None = None, weights: Weights | None = None):
        self.budget = budget_tokens
        self.count = count_tokens or (lambda s: max(1, len(s) // 4))
        self.layout = layout or Layout()
        self.w = weights or Weights()

    def _tokens(self, msg: dict) -> int:
        return self.count(_text(msg)) + 4   # role / framing tokens

    def plan(self, messages: list[dict]) -> Plan:
        n = len(messages)
        L = self.layout
        areas = []
        first_current = max(0, n - L.current_n)
        first_recent = max(0, first_current - L.recent_n)
        for i, m in enumerate(messages):
            if m.get("role") in ("system", "developer"):
                areas.append("base")
            elif i >= first_current:
                areas.append("current")
            elif i >= first_recent:
                areas.append("recent")
            else:
                areas.append("deep")
        toks = [self._tokens(m) for m in messages]
        # forecast: what the current turn talks about
        forecast = _terms(" ".join(_text(messages[i]) for i in range(first_current, n)))
        docs = [set(_terms(_text(m))) for m in messages]
        df: dict[str, int] = {}
        for d in docs:
            for t in d:
                df[t] = df.get(t, 0) + 1
        idf = {t: math.log((n + 1) / (c + 0.5)) for t, c in df.items()}
        fset = set(forecast)
        later_text = [set() for _ in range(n)]
        acc: set[str] = set()
        for i in range(n - 1, -1, -1):
            later_text[i] = set(acc)
            acc |= docs[i]
        benefit = []
        for i, m in enumerate(messages):
            rel = sum(idf.get(t, 0.0) for t in docs[i] & fset) / (1.0 + math.sqrt(len(docs[i]) or 1))
            rec = 0.5 ** ((n - 1 - i) / self.w.half_life)
            referenced = len(docs[i] & later_text[i]) / (len(docs[i]) or 1) if m.get("role") == "tool" else 0.0
            dur = 1.0 if m.get("role") in ("system", "developer") else referenced
            benefit.append(self.w.relevance * rel + self.w.recency * rec + self.w.durability * dur)
        resident = [a in ("base", "current") for a in areas]
        used = sum(t for t, r in zip(toks, resident) if r)
        # recent: newest first while they fit (exact precision)
        for i in range(first_current - 1, first_recent - 1, -1):
            if areas[i] == "recent" and used + toks[i] <= self.budget:
                resident[i] = True
                used += toks[i]
        # deep: budgeted 0/1 knapsack on the remaining budget (bucketed token costs)
        deep = [i for i, a in enumerate(areas) if a == "deep"]
        ptr_cost = 12   # a pointer line in place of an elided cell
        room = self.budget - used - ptr_cost * len(deep)
        if deep and room > 0:
            g = L.granule
            cap = room // g
            cost = [max(1, math.ceil((toks[i] - ptr_cost) / g)) for i in deep]
            best = [0.0] * (cap + 1)
            take = [[False] * (cap + 1) for _ in deep]
            for k, i in enumerate(deep):
                c = cost[k]
                for w in range(cap, c - 1, -1):
                    v = best[w - c] + benefit[i]
                    if v > best[w]:
                        best[w] = v
                        take[k][w] = True
            w = cap
            for k in range(len(deep) - 1, -1, -1):
                if take[k][w]:
                    resident[deep[k]] = True
                    w -= cost[k]
            used += sum(toks[i] - ptr_cost for k, i in enumerate(deep) if resident[i])
        used += ptr_cost * sum(1 for i in deep if not resident[i])
        out = []
        for i, m in enumerate(messages):
            if resident[i]:
                out.append(m)
            else:
                out.append({"role": m.get("role", "user"),
                            "content": f"[elided cell {i}: {m.get('role', 'message')}, {toks[i]} tokens; "
                                       f"page in by id {i}]"})
        cells = [CellPlan(i, areas[i], toks[i], round(benefit[i], 4), resident[i]) for i in range(n)]
        return Plan(cells, self.budget, used, out)
