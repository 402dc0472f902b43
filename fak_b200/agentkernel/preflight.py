"""Pre-flight rungs: cheapest-first well-formedness checks of a tool call before it is adjudicated
by the policy, so a malformed call is refused before anything runs.

* rung 0 -- static parse: the arguments are a JSON object (raw strings that failed to parse
  arrive as ``{"__raw__": ...}``);
* rung 1 -- schema: required fields present and scalar types right, against a minimal JSON Schema
  ({"type": "object", "properties": {name: {"type": ...}}, "required": [...]}) registered per
  tool (e.g. from the tool list of a chat request).

A failed rung is a DENY (reason MALFORMED) with the rung number in its meta; a call that
passes every rung gets DEFER (nothing to prove here) and goes on to the policy.  Each catch is
counted per rung.

Reference: internal/preflight/preflight.go:1-286 (rung 0 static parse, rung 1 schema check,
registered as a low-rank adjudicator whose deny wins the fold).
"""
from __future__ import annotations

import threading

from .abi import Reason, ToolCall, Verdict, VerdictKind

_TYPES = {"string": (str,), "integer": (int,), "number": (int, float), "boolean": (bool,), "object": (dict,),
          "array": (list,), "null": (type(None),)}


def _type_ok(value, t: str | list) -> bool:
    ts = t if isinstance(t, list) else [t]
    for name in ts:
        py = _TYPES.get(name)
        if py is None:
            return True   # unknown type keywords are not checked
        if isinstance(value, bool) and name in ("integer", "number"):
            continue      # bool is not a number in JSON Schema
        if isinstance(value, py):
            return True
    return False


class Preflight:
    def __init__(self):
        self.schemas: dict[str, dict] = {}
        self.catches = {0: 0, 1: 0}
        self._lock = threading.Lock()

    def register_schema(self, tool: str, schema: dict) -> None:
        self.schemas[tool] = schema

    def register_openai_tools(self, tools: list[dict]) -> None:
        """Schemas from an OpenAI ``tools`` list ({"type": "function", "function": {name, parameters}})."""
        for t in tools or []:
            fn = t.get("function", t)
            if fn.get("name") and isinstance(fn.get("parameters"), dict):
                self.register_schema(fn["name"], fn["parameters"])

    def _deny(self, rung: int, claim: str) -> Verdict:
        with self._lock:
            self.catches[rung] += 1
        return Verdict(VerdictKind.DENY, Reason.MALFORMED, by="preflight", claim=claim, meta={"rung": rung})

    def check(self, call: ToolCall) -> Verdict:
        args = call.args
        if not isinstance(args, dict) or "__raw__" in args:
            return self._deny(0, "arguments are not a JSON object")
        schema = self.schemas.get(call.tool)
        if schema:
            props = schema.get("properties", {}) or {}
            for req in schema.get("required", []) or []:
                if req not in args:
                    return self._deny(1, f"missing required field {req!r}")
            for k, v in args.items():
                spec = props.get(k)
                if isinstance(spec, dict) and "type" in spec and not _type_ok(v, spec["type"]):
                    return self._deny(1, f"field {k!r} is not {spec['type']}")
                if isinstance(spec, dict) and "enum" in spec and v not in spec["enum"]:
                    return self._deny(1, f"field {k!r} is not one of {spec['enum']}")
            if schema.get("additionalProperties") is False:
                extra = [k for k in args if k not in props]
                if extra:
                    return self._deny(1, f"unexpected field {extra[0]!r}")
        return Verdict(VerdictKind.DEFER, Reason.NONE, by="preflight")
