"""Serving autoscaler signals and the scale planner for prefill / decode replica pools.

``SignalWindow`` folds completed requests (TTFT, TPOT) and the engine's queue depth and KV-page
use into the planner's signal set: goodput (the fraction of recent requests that met both the TTFT
and the TPOT objective), queue depth, KV utilisation, and the window's p50 TTFT / TPOT.
``ServingAutoscaler.plan`` turns a pool's signals into a decision against a ``PoolObjective``:
scale up by ``scale_step`` when any high signal fires (queue high, goodput below target, KV use
high, TTFT or TPOT over its objective), scale down when every signal is low, otherwise hold --
bounded by min/max replicas, gated by ``hysteresis_ticks`` consecutive ticks in the same direction
and a ``cooldown_s`` after each action.  In ``defer`` mode (an external planner owns the replica
count) the decision is recorded with action "deferred".  The planner only decides; starting or
draining replicas is the host's job (``serve/router.py`` holds the replica set).

Reference behaviour: internal/gateway/serving_autoscaler.go:37-615 (PoolSignals, PoolObjective,
high/low reason sets, hysteresis and cooldown, native vs delegated mode).
"""
from __future__ import annotations

import collections
import dataclasses
import statistics
import time


@dataclasses.dataclass
class PoolSignals:
    goodput: float = 1.0
    queue_depth: int = 0
    kv_utilization: float = 0.0
    ttft_s: float = 0.0
    tpot_s: float = 0.0


@dataclasses.dataclass
class PoolObjective:
    min_replicas: int = 1
    max_replicas: int = 8
    scale_step: int = 1
    goodput_target: float = 0.9
    queue_high: int = 16
    queue_low: int = 0
    kv_util_high: float = 0.9
    kv_util_low: float = 0.5
    ttft_slo_s: float = 0.5
    tpot_slo_s: float = 0.05

    def high_reasons(self, s: PoolSignals) -> list[str]:
        r = []
        if self.queue_high > 0 and s.queue_depth > self.queue_high:
            r.append("queue_high")
        if self.goodput_target > 0 and s.goodput < self.goodput_target:
            r.append("goodput_below_target")
        if self.kv_util_high > 0 and s.kv_utilization > self.kv_util_high:
            r.append("kv_util_high")
        if self.ttft_slo_s > 0 and s.ttft_s > self.ttft_slo_s:
            r.append("ttft_slo")
        if self.tpot_slo_s > 0 and s.tpot_s > self.tpot_slo_s:
            r.append("tpot_slo")
        return r

    def low_enough(self, s: PoolSignals) -> bool:
        return (s.queue_depth <= self.queue_low
                and not (self.goodput_target > 0 and s.goodput < self.goodput_target)
                and not (self.kv_util_low > 0 and s.kv_utilization > self.kv_util_low)
                and not (self.ttft_slo_s > 0 and s.ttft_s > self.ttft_slo_s)
                and not (self.tpot_slo_s > 0 and s.tpot_s > self.tpot_slo_s))


class SignalWindow:
    """The last ``size`` completed requests plus live gauges, folded into PoolSignals."""

    def __init__(self, objective: PoolObjective, size: int = 256):
        self.obj = objective
        self.done: collections.deque = collections.deque(maxlen=size)

    def observe(self, ttft_s: float | None, tpot_s: float | None) -> None:
        self.done.append((ttft_s, tpot_s))

    def signals(self, queue_depth: int = 0, kv_utilization: float = 0.0) -> PoolSignals:
        if not self.done:
            return PoolSignals(1.0, queue_depth, kv_utilization, 0.0, 0.0)
        o = self.obj
        good = sum(1 for t, p in self.done
                   if (t is None or o.ttft_slo_s <= 0 or t <= o.ttft_slo_s)
                   and (p is None or o.tpot_slo_s <= 0 or p <= o.tpot_slo_s))
        ttfts = [t for t, _ in self.done if t is not None]
        tpots = [p for _, p in self.done if p is not None]
        return PoolSignals(good / len(self.done), queue_depth, kv_utilization,
                           statistics.median(ttfts) if ttfts else 0.0, statistics.median(tpots) if tpots else 0.0)


@dataclasses.dataclass
class ScaleDecision:
    pool: str
    action: str                 # hold | scale_up | scale_down | deferred
    current: int
    desired: int
    reasons: list[str]
    signals: PoolSignals

    def to_dict(self) -> dict:
        d = dataclasses.asdict(self)
        return d


class ServingAutoscaler:
    def __init__(self, objectives: dict[str, PoolObjective], mode: str = "native", cooldown_s: float = 60.0,
                 hysteresis_ticks: int = 2, clock=time.monotonic):
        if mode not in ("native", "defer"):
            raise ValueError("mode must be 'native' or 'defer'")
        self.obj = objectives
        self.mode = mode
        self.cooldown_s = cooldown_s
        self.hysteresis = max(1, hysteresis_ticks)
        self.clock = clock
        self._pending: dict[str, tuple[int, int]] = {}     # pool -> (direction, consecutive ticks)
        self._last_action: dict[str, float] = {}
        self.history: list[ScaleDecision] = []

    def _target(self, pool: str, current: int, s: PoolSignals) -> tuple[int, list[str]]:
        o = self.obj[pool]
        high = o.high_reasons(s)
        if high:
            return min(o.max_replicas, current + o.scale_step), high
        if o.low_enough(s) and current > o.min_replicas:
            return max(o.min_replicas, current - o.scale_step), ["all_signals_low"]
        return max(o.min_replicas, min(o.max_replicas, current)), ["within_band"]

    def plan(self, pool: str, current: int, s: PoolSignals) -> ScaleDecision:
        target, reasons = self._target(pool, current, s)
        d = ScaleDecision(pool, "hold", current, target, list(reasons), s)
        if self.mode == "defer":
            d.action = "deferred"
            d.reasons.append("external_planner")
        else:
            dirn = (target > current) - (target < current)
            if dirn == 0:
                self._pending.pop(pool, None)
                d.desired = current
            else:
                pd, n = self._pending.get(pool, (0, 0))
                n = n + 1 if pd == dirn else 1
                self._pending[pool] = (dirn, n)
                now = self.clock()
                if n < self.hysteresis:
                    d.reasons.append(f"hysteresis_{n}/{self.hysteresis}")
                    d.desired = current
                elif now - self._last_action.get(pool, -1e18) < self.cooldown_s:
                    d.reasons.append("cooldown")
                    d.desired = current
                else:
                    d.action = "scale_up" if dirn > 0 else "scale_down"
                    self._last_action[pool] = now
                    self._pending.pop(pool, None)
        self.history.append(d)
        return d
