"""The agent kernel: adjudicate -> dispatch -> admit -> journal, for every tool call.

``Kernel.syscall`` is the synchronous path; ``submit``/``reap`` the asynchronous one
(reference: internal/kernel/kernel.go:132-640 -- Decide, Fold, AdmitResult, Submit, Reap,
Syscall).  Tools execute through registered in-process handlers (the reference's vDSO tier);
a call with no handler is only adjudicated (the wrapped agent executes it itself and the
gateway reports the verdict).
"""
from __future__ import annotations

import concurrent.futures
import threading
import time
from typing import Any, Callable

from .abi import Reason, Result, Status, ToolCall, Verdict, VerdictKind
from .adjudicator import Adjudicator
from .ctxmmu import ContextMMU
from .grammar import GrammarRung
from .journal import Journal
from .policy import Policy
from .preflight import Preflight
from .vdso import VDSO

Handler = Callable[[dict], Any]


class Kernel:
    def __init__(self, policy: Policy | None = None, journal_path: str | None = None, mmu: ContextMMU | None = None,
                 workers: int = 4, preflight: Preflight | None = None, vdso: VDSO | None = None,
                 grammar: GrammarRung | None = None):
        self.grammar = grammar or GrammarRung()
        self.preflight = preflight or Preflight()
        self.vdso = vdso or VDSO()
        self.adjudicator = Adjudicator(policy)
        self.journal = Journal(journal_path)
        self.mmu = mmu or ContextMMU()
        self.handlers: dict[str, Handler] = {}
        self._pool = concurrent.futures.ThreadPoolExecutor(max_workers=workers)
        self._pending: dict[int, concurrent.futures.Future] = {}
        self._lock = threading.Lock()
        self.stats = {"allow": 0, "deny": 0, "transform": 0, "quarantine": 0, "decide_ns": 0, "calls": 0}

    def register(self, tool: str, handler: Handler) -> None:
        self.handlers[tool] = handler

    def set_policy(self, p: Policy) -> None:
        self.adjudicator.set_policy(p)
        self.journal.append("policy_reload")

    def decide(self, call: ToolCall) -> Verdict:
        t0 = time.perf_counter_ns()
        # the grammar rung first (cheapest): a mis-shaped call is repaired in place or refused
        g = self.grammar.check(call)
        if g.kind == VerdictKind.DENY:
            v = g
        else:
            checked = call
            if g.kind == VerdictKind.TRANSFORM:   # the repaired call goes through every later rung
                checked = ToolCall(call.tool, g.new_args, call.op, call.engine, call.seq, call.trace_id, call.meta)
            v = self.preflight.check(checked)       # malformed calls never reach the policy
            if v.kind == VerdictKind.DEFER:
                v = self.adjudicator.adjudicate(checked)
            if g.kind == VerdictKind.TRANSFORM and v.kind == VerdictKind.ALLOW:
                v = Verdict(VerdictKind.TRANSFORM, Reason.MISROUTE, by=f"grammar+{v.by}", claim=v.claim,
                            new_args=g.new_args, meta={**g.meta, **v.meta})
        dt = time.perf_counter_ns() - t0
        with self._lock:
            self.stats["calls"] += 1
            self.stats["decide_ns"] += dt
            key = {VerdictKind.ALLOW: "allow", VerdictKind.TRANSFORM: "transform",
                   VerdictKind.QUARANTINE: "quarantine"}.get(v.kind, "deny")
            self.stats[key] += 1
        self.journal.record_decision(call, v)
        return v

    def _execute(self, call: ToolCall, verdict: Verdict) -> Result:
        args = verdict.new_args if verdict.kind == VerdictKind.TRANSFORM and verdict.new_args is not None else call.args
        hit, out, tier = self.vdso.lookup(call.tool, args)
        if hit:   # answered by the fast path: the same result a fresh call gives
            self.journal.append("vdso_hit", tool=call.tool, seq=call.seq, tier=tier)
            return Result(call, out, Status.OK, verdict)
        h = self.handlers.get(call.tool)
        if h is None:
            return Result(call, None, Status.ERROR, Verdict(VerdictKind.DENY, Reason.UNKNOWN_TOOL, by="kernel",
                                                             claim=call.tool))
        try:
            out = h(args)
        except Exception as e:  # a failing tool is a result, not a kernel crash
            return Result(call, f"{type(e).__name__}: {e}", Status.ERROR, verdict)
        adm = self.mmu.admit(call.tool, out if isinstance(out, str) else str(out))
        # the cache holds what the model was shown (the admitted content), never a raw result
        self.vdso.complete(call.tool, args, adm.content, cacheable=adm.verdict.kind != VerdictKind.DENY)
        self.journal.append("admission", tool=call.tool, seq=call.seq, verdict=adm.verdict.to_dict(),
                            findings=len(adm.findings))
        if adm.verdict.kind == VerdictKind.DENY:
            return Result(call, None, Status.ERROR, adm.verdict)
        return Result(call, adm.content, Status.OK, adm.verdict if adm.verdict.kind != VerdictKind.ALLOW else verdict)

    def syscall(self, call: ToolCall) -> Result:
        v = self.decide(call)
        if not v.allowed:
            return Result(call, None, Status.ERROR, v)
        return self._execute(call, v)

    def submit(self, call: ToolCall) -> Result:
        v = self.decide(call)
        if not v.allowed:
            return Result(call, None, Status.ERROR, v)
        fut = self._pool.submit(self._execute, call, v)
        with self._lock:
            self._pending[call.seq] = fut
        return Result(call, None, Status.PENDING, v)

    def reap(self, timeout: float | None = None) -> list[Result]:
        with self._lock:
            futs = dict(self._pending)
        done, _ = concurrent.futures.wait(list(futs.values()), timeout=timeout)
        out = []
        with self._lock:
            for seq, f in list(self._pending.items()):
                if f in done:
                    out.append(f.result())
                    del self._pending[seq]
        return out

    def shutdown(self) -> None:
        self._pool.shutdown(wait=True)
