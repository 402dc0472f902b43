"""The agent-kernel syscall ABI: tool calls, verdicts, results, refusal reasons.

Every tool call a model proposes becomes a ``ToolCall``; the kernel adjudicates it into a
``Verdict`` before anything runs.  The verdict kinds and refusal reason names are the
reference's closed vocabulary (internal/abi/types.go:160-330, internal/abi/reasons.go:12-45),
kept identical because journals, policies and clients exchange them by name.
"""
from __future__ import annotations

import dataclasses
import enum
import itertools
import json
import time
from typing import Any


class VerdictKind(enum.IntEnum):
    ALLOW = 0
    DENY = 1
    TRANSFORM = 2        # rewrite the arguments (payload: new args)
    QUARANTINE = 3       # hold the RESULT out of the model context
    REQUIRE_WITNESS = 4  # gate pending an independent read-back
    DEFER = 5            # not adjudicable here; pass to the next link
    INDETERMINATE = 6    # undecided cheaply; fail closed


class Reason(enum.IntEnum):
    NONE = 0
    DEFAULT_DENY = 1
    POLICY_BLOCK = 2
    SELF_MODIFY = 3
    LEASE_HELD = 4
    TRUST_VIOLATION = 5
    MALFORMED = 6
    MISROUTE = 7
    RATE_LIMITED = 8
    SECRET_EXFIL = 9
    UNWITNESSED = 10
    OVERSIZE = 11
    UNKNOWN_TOOL = 12
    RESULT_SECRET_DISCOVERED = 13
    EGRESS_BLOCK = 14

    @classmethod
    def parse(cls, s: str | int) -> "Reason":
        if isinstance(s, int):
            return cls(s)
        return cls[s.strip().upper()]


class Status(enum.IntEnum):
    OK = 0
    ERROR = 1
    PENDING = 2


_seq = itertools.count(1)


@dataclasses.dataclass
class ToolCall:
    tool: str
    args: dict[str, Any] = dataclasses.field(default_factory=dict)
    op: str = "call"
    engine: str = ""
    seq: int = dataclasses.field(default_factory=lambda: next(_seq))
    trace_id: str = ""
    meta: dict[str, str] = dataclasses.field(default_factory=dict)

    def to_dict(self) -> dict:
        return {"tool": self.tool, "args": self.args, "op": self.op, "seq": self.seq, "trace_id": self.trace_id,
                "meta": self.meta}

    @classmethod
    def from_dict(cls, d: dict) -> "ToolCall":
        args = d.get("args", d.get("arguments", {}))
        if isinstance(args, str):
            try:
                args = json.loads(args) if args else {}
            except json.JSONDecodeError:
                args = {"__raw__": args}
        return cls(tool=str(d.get("tool", d.get("name", ""))), args=args if isinstance(args, dict) else {"value": args},
                   op=d.get("op", "call"), trace_id=d.get("trace_id", ""), meta=dict(d.get("meta", {})))


@dataclasses.dataclass
class Verdict:
    kind: VerdictKind
    reason: Reason = Reason.NONE
    by: str = ""
    claim: str = ""                      # bounded witness (never the whole policy, never arg values)
    new_args: dict[str, Any] | None = None  # TRANSFORM payload
    meta: dict[str, str] = dataclasses.field(default_factory=dict)

    @property
    def allowed(self) -> bool:
        return self.kind in (VerdictKind.ALLOW, VerdictKind.TRANSFORM)

    def to_dict(self) -> dict:
        d = {"kind": self.kind.name, "reason": self.reason.name, "by": self.by}
        if self.claim:
            d["claim"] = self.claim
        if self.meta:
            d["meta"] = self.meta
        if self.new_args is not None:
            d["transformed"] = True
        return d


@dataclasses.dataclass
class Result:
    call: ToolCall
    payload: Any = None
    status: Status = Status.OK
    verdict: Verdict | None = None
    meta: dict[str, str] = dataclasses.field(default_factory=dict)
    ts: float = dataclasses.field(default_factory=time.time)
