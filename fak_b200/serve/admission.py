"""Gateway admission control: a running-set cap, a token budget, priority with aging, and shedding.

Requests are *offered* to the controller, which either admits them into the running set at once,
queues them, sheds them (the waiting queue is full: HTTP 429) or denies them (a per-tenant trust
verdict: HTTP 403).  ``schedule`` promotes waiting requests in effective-priority order while the
running set has headroom: at most ``max_num_seqs`` requests and ``token_budget`` tokens (prompt +
planned decode) in flight.  Lower priority values go first; a waiting request's effective priority
improves by one for every ``aging_rounds`` scheduling rounds it is passed over, so a flood of
higher-priority arrivals cannot starve it.  Ties go to the older arrival, then the trace id, so
the admission order is a deterministic function of the offers (no clock, no randomness).

``lease`` is the request-path wrapper: a served request holds a lease while it generates; the
lease blocks (bounded) until the request is admitted and releases its budget on exit.

Reference behaviour: internal/gateway/admission.go:71-682 (AdmissionPolicy, Offer / Schedule,
aging starvation guard, VerdictShed -> 429, VerdictDenied), written here from that description.
"""
from __future__ import annotations

import dataclasses
import enum
import threading
import time
from contextlib import contextmanager


class Verdict(enum.Enum):
    ADMITTED = "admitted"
    QUEUED = "queued"
    SHED = "shed"
    DENIED = "denied"


@dataclasses.dataclass
class AdmissionPolicy:
    max_num_seqs: int = 256        # running-set cap (<= 0: none)
    token_budget: int = 8192 * 16  # sum of running footprints (<= 0: none)
    max_waiting: int = 1024        # waiting-queue bound before shedding (<= 0: unbounded)
    aging_rounds: int = 1          # rounds passed over per priority step gained (<= 0: no aging)


@dataclasses.dataclass
class SeqRequest:
    trace_id: str
    priority: int = 0
    tokens: int = 0
    deny: bool = False             # per-tenant trust verdict
    deny_reason: str = ""
    # bookkeeping
    round_enqueued: int = 0
    seq: int = 0


class AdmissionError(Exception):
    def __init__(self, verdict: Verdict, msg: str, status: int):
        super().__init__(msg)
        self.verdict, self.status = verdict, status


class AdmissionController:
    def __init__(self, policy: AdmissionPolicy | None = None):
        self.policy = policy or AdmissionPolicy()
        self.running: dict[str, SeqRequest] = {}
        self.waiting: list[SeqRequest] = []
        self.round = 0
        self._seq = 0
        self.counts = {"admitted": 0, "queued": 0, "shed": 0, "denied": 0, "released": 0}
        self._cv = threading.Condition()

    # ---------------------------------------------------------------- policy (pure, deterministic)
    def _tokens_running(self) -> int:
        return sum(r.tokens for r in self.running.values())

    def _fits(self, r: SeqRequest) -> bool:
        p = self.policy
        if p.max_num_seqs > 0 and len(self.running) >= p.max_num_seqs:
            return False
        if p.token_budget > 0 and self.running and self._tokens_running() + r.tokens > p.token_budget:
            return False   # an oversized request still runs alone rather than never
        return True

    def effective_priority(self, r: SeqRequest) -> int:
        a = self.policy.aging_rounds
        passed = self.round - r.round_enqueued
        return r.priority - (passed // a if a > 0 else 0)

    def _order(self, r: SeqRequest):
        return (self.effective_priority(r), r.round_enqueued, r.seq, r.trace_id)

    def offer(self, r: SeqRequest) -> Verdict:
        """Classify one request: admitted now, queued, shed or denied."""
        with self._cv:
            self._seq += 1
            r.seq = self._seq
            r.round_enqueued = self.round
            if r.deny:
                self.counts["denied"] += 1
                return Verdict.DENIED
            if not self.waiting and self._fits(r):
                self.running[r.trace_id] = r
                self.counts["admitted"] += 1
                return Verdict.ADMITTED
            if self.policy.max_waiting > 0 and len(self.waiting) >= self.policy.max_waiting:
                self.counts["shed"] += 1
                return Verdict.SHED
            self.waiting.append(r)
            self.counts["queued"] += 1
            return Verdict.QUEUED

    def schedule(self) -> list[str]:
        """One scheduling round: promote waiting requests in effective-priority order while they fit;
        returns the admitted trace ids."""
        with self._cv:
            self.round += 1
            out = []
            self.waiting.sort(key=self._order)
            while self.waiting and self._fits(self.waiting[0]):
                r = self.waiting.pop(0)
                self.running[r.trace_id] = r
                self.counts["admitted"] += 1
                out.append(r.trace_id)
            if out:
                self._cv.notify_all()
            return out

    def release(self, trace_id: str) -> None:
        with self._cv:
            if self.running.pop(trace_id, None) is not None:
                self.counts["released"] += 1
            self.waiting = [r for r in self.waiting if r.trace_id != trace_id]
        self.schedule()

    def snapshot(self) -> dict:
        with self._cv:
            return {"running": len(self.running), "waiting": len(self.waiting),
                    "running_tokens": self._tokens_running(), "round": self.round, **self.counts}

    # ---------------------------------------------------------------- request-path lease
    @contextmanager
    def lease(self, r: SeqRequest, timeout_s: float = 60.0):
        """Hold an admission lease around one served request (raises AdmissionError when shed,
        denied, or not admitted within ``timeout_s``)."""
        v = self.offer(r)
        if v == Verdict.SHED:
            raise AdmissionError(v, "server overloaded: waiting queue full", 429)
        if v == Verdict.DENIED:
            raise AdmissionError(v, f"admission denied: {r.deny_reason or 'tenant policy'}", 403)
        if v == Verdict.QUEUED:
            self.schedule()
            deadline = time.monotonic() + timeout_s
            with self._cv:
                while r.trace_id not in self.running:
                    left = deadline - time.monotonic()
                    if left <= 0:
                        self.waiting = [w for w in self.waiting if w.trace_id != r.trace_id]
                        self.counts["shed"] += 1
                        raise AdmissionError(Verdict.SHED, "admission wait timed out", 429)
                    self._cv.wait(left)
        try:
            yield r
        finally:
            self.release(r.trace_id)
