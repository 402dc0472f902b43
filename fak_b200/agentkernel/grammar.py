"""The grammar rung: a tool call's argument SHAPE, checked (and where the fix is mechanical,
repaired) before the call runs -- the well-formedness axis the policy rungs cannot see.

* ``GrammarRung`` holds one grammar (ordered named parameters plus synonym aliases) per tool,
  deduplicated by content digest so a grammar learned once is one entry however many tools share
  it.  ``check`` gives:

  - no grammar for the tool                 -> DEFER (fail-open: never over-refuse);
  - every required parameter present        -> DEFER;
  - an alias rename closes the gap          -> TRANSFORM (reason MISROUTE, the renamed arguments);
  - positional arguments (``_positional``)
    whose count equals the grammar's arity   -> TRANSFORM (zipped onto the parameter names);
  - anything else                           -> DENY (MISROUTE: the model can fix it).

  A parameter counts as present under its name or as ``named:<name>``.  Grammars come from
  ``add`` or from an MCP-style JSON Schema (``load_json_schema``: properties in sorted order).
* ``TypeRegistry`` -- message types for agent-to-agent payloads: a type is a field set (sorted by
  name, deduplicated by digest); ``validate`` lists missing required fields, ``pack`` wraps a
  valid payload in ``{"type", "digest", "payload"}`` and ``unpack`` accepts only an envelope whose
  digest matches the registered type and whose payload is valid.
* Durability -- how long a memory write may be believed, a closed vocabulary (turn, session,
  durable, bounded) and a fail-closed promotion predicate: only a write stamped ``durable``
  promotes to a longer-lived tier; in ``warn`` mode the refusal is recorded but the write still
  persists, in ``enforce`` mode it does not.  The class is an input stamped at write time, never
  inferred from the content.

Reference: internal/grammar/grammar.go:45-270 (rung, aliases, positional repair, JSON Schema),
msgtype.go:33-190 (message types), durability.go:31-203 (vocabulary and promotion).
"""
from __future__ import annotations

import dataclasses
import enum
import hashlib
import json
import threading
from typing import Any

from .abi import Reason, ToolCall, Verdict, VerdictKind


@dataclasses.dataclass(frozen=True)
class Param:
    name: str
    type: str = ""
    required: bool = False

    def to_dict(self) -> dict:
        return {"name": self.name, "type": self.type, "required": self.required}


@dataclasses.dataclass(frozen=True)
class Grammar:
    params: tuple[Param, ...]
    aliases: tuple[tuple[str, str], ...] = ()   # (synonym key, canonical parameter), sorted

    @classmethod
    def of(cls, params: list[Param] | tuple[Param, ...], aliases: dict[str, str] | None = None) -> "Grammar":
        return cls(tuple(params), tuple(sorted((aliases or {}).items())))

    def digest(self) -> str:
        doc = {"params": [p.to_dict() for p in self.params], "aliases": dict(self.aliases)}
        return hashlib.sha256(json.dumps(doc, sort_keys=True, separators=(",", ":")).encode()).hexdigest()[:24]

    def missing(self, args: dict) -> list[str]:
        """Required parameters absent from the arguments (present as ``name`` or ``named:name``)."""
        return [p.name for p in self.params if p.required and p.name not in args and f"named:{p.name}" not in args]


def _renamed(args: dict, aliases: dict[str, str]) -> tuple[dict, bool]:
    """The arguments with every synonym key renamed to its canonical parameter when the canonical
    one is not already there; whether anything was renamed."""
    out: dict = {}
    renamed = False
    for k, v in args.items():
        canon = aliases.get(k)
        if canon is not None and canon not in args:
            out[canon] = v
            renamed = True
        else:
            out[k] = v
    return out, renamed


class GrammarRung:
    name = "grammar"

    def __init__(self):
        self._by_tool: dict[str, str] = {}
        self._by_digest: dict[str, Grammar] = {}
        self._lock = threading.Lock()
        self.repairs = 0
        self.denies = 0

    def add(self, tool: str, g: Grammar) -> None:
        d = g.digest()
        with self._lock:
            self._by_digest.setdefault(d, g)
            self._by_tool[tool] = d

    def has(self, tool: str) -> bool:
        return tool in self._by_tool

    def unique_grammars(self) -> int:
        return len(self._by_digest)

    def grammar(self, tool: str) -> Grammar | None:
        d = self._by_tool.get(tool)
        return self._by_digest.get(d) if d is not None else None

    def load_json_schema(self, tool: str, schema: dict | str | bytes, aliases: dict[str, str] | None = None) -> None:
        """A grammar from {"properties": {name: {"type": ...}}, "required": [...]} (parameters in
        sorted name order, so the same schema always gives the same grammar)."""
        doc = json.loads(schema) if isinstance(schema, (str, bytes)) else schema
        props = doc.get("properties") or {}
        req = set(doc.get("required") or [])
        params = [Param(n, str((props[n] or {}).get("type", "")), n in req) for n in sorted(props)]
        self.add(tool, Grammar.of(params, aliases))

    def register_openai_tools(self, tools: list[dict] | None) -> None:
        """Grammars from an OpenAI ``tools`` list (each function's ``parameters`` JSON Schema)."""
        for t in tools or []:
            fn = t.get("function", t) if isinstance(t, dict) else {}
            if fn.get("name") and isinstance(fn.get("parameters"), dict):
                self.load_json_schema(fn["name"], fn["parameters"])

    def check(self, call: ToolCall) -> Verdict:
        g = self.grammar(call.tool)
        if g is None:
            return Verdict(VerdictKind.DEFER, by=self.name)
        args = call.args if isinstance(call.args, dict) else {}
        if not g.missing(args):
            return Verdict(VerdictKind.DEFER, by=self.name)
        if g.aliases:
            fixed, renamed = _renamed(args, dict(g.aliases))
            if renamed and not g.missing(fixed):
                return self._repair(fixed, "alias")
        pos = args.get("_positional")
        if isinstance(pos, list) and len(pos) == len(g.params):
            return self._repair({p.name: v for p, v in zip(g.params, pos)}, "positional")
        with self._lock:
            self.denies += 1
        return Verdict(VerdictKind.DENY, Reason.MISROUTE, by=self.name,
                       claim=f"missing {','.join(g.missing(args))}")

    def _repair(self, new_args: dict, how: str) -> Verdict:
        with self._lock:
            self.repairs += 1
        return Verdict(VerdictKind.TRANSFORM, Reason.MISROUTE, by=self.name, new_args=new_args, meta={"repair": how})

    def stats(self) -> dict:
        return {"repairs": self.repairs, "denies": self.denies, "grammars": self.unique_grammars(),
                "tools": len(self._by_tool)}


# ---- message types ---------------------------------------------------------------------------
@dataclasses.dataclass(frozen=True)
class MessageType:
    name: str
    fields: tuple[Param, ...]
    digest: str


class TypeRegistry:
    def __init__(self):
        self._by_name: dict[str, str] = {}
        self._by_digest: dict[str, MessageType] = {}
        self._lock = threading.Lock()

    def register(self, name: str, fields: list[Param]) -> MessageType:
        fs = tuple(sorted(fields, key=lambda p: p.name))
        d = Grammar(fs).digest()
        with self._lock:
            first = self._by_digest.setdefault(d, MessageType(name, fs, d))
            self._by_name[name] = d
        return MessageType(name, first.fields, d)

    def lookup(self, name: str) -> MessageType | None:
        d = self._by_name.get(name)
        t = self._by_digest.get(d) if d is not None else None
        return MessageType(name, t.fields, t.digest) if t is not None else None

    def lookup_digest(self, digest: str) -> MessageType | None:
        return self._by_digest.get(digest)

    def unique_types(self) -> int:
        return len(self._by_digest)

    def validate(self, name: str, payload: dict) -> tuple[list[str], bool]:
        """(missing required fields, whether the type is known)."""
        t = self.lookup(name)
        if t is None:
            return [], False
        return Grammar(t.fields).missing(payload), True

    def pack(self, name: str, payload: dict) -> bytes | None:
        missing, known = self.validate(name, payload)
        if not known or missing:
            return None
        t = self.lookup(name)
        return json.dumps({"type": name, "digest": t.digest, "payload": payload}).encode()

    def unpack(self, data: bytes | str) -> tuple[str, dict] | None:
        try:
            env = json.loads(data)
        except (ValueError, TypeError):
            return None
        if not isinstance(env, dict) or not isinstance(env.get("payload"), dict):
            return None
        t = self.lookup(str(env.get("type", "")))
        if t is None or env.get("digest") != t.digest:
            return None
        missing, _ = self.validate(t.name, env["payload"])
        return None if missing else (t.name, env["payload"])


# ---- durability of memory writes -------------------------------------------------------------
DURABILITY = ("durable", "session", "bounded", "turn")   # the closed vocabulary, most durable first


def known_durability(cls: str) -> bool:
    return cls in DURABILITY


class PromotionMode(enum.Enum):
    WARN = "warn"
    ENFORCE = "enforce"


@dataclasses.dataclass(frozen=True)
class PromotionVerdict:
    cls: str
    known: bool
    promote: bool
    mode: PromotionMode
    reason: str = ""

    def should_persist(self) -> bool:
        """Enforce mode persists only a promotable write; warn mode persists and only records."""
        return self.promote if self.mode is PromotionMode.ENFORCE else True

    def would_refuse(self) -> bool:
        return not self.promote


def may_promote(cls: str, mode: PromotionMode = PromotionMode.WARN) -> PromotionVerdict:
    """Only a write stamped ``durable`` may move to a longer-lived tier; an unknown or missing
    class fails closed like a refusal."""
    if not known_durability(cls):
        return PromotionVerdict(cls, False, False, mode, "unknown_class")
    if cls == "durable":
        return PromotionVerdict(cls, True, True, mode)
    return PromotionVerdict(cls, True, False, mode, "non_durable")
