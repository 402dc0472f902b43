"""The grammar rung (argument-shape check and mechanical repair), message types and the durability
promotion predicate; the rung inside the kernel's decision chain."""
from fak_b200.agentkernel.abi import Reason, Status, ToolCall, VerdictKind
from fak_b200.agentkernel.grammar import (Grammar, GrammarRung, Param, PromotionMode, TypeRegistry, known_durability,
                                          may_promote)
from fak_b200.agentkernel.kernel import Kernel
from fak_b200.agentkernel.policy import policy_from_dict

FX = Grammar.of([Param("from_currency", "string", True), Param("to_currency", "string", True),
                 Param("amount", "number", False)], {"from": "from_currency", "to": "to_currency"})


def test_well_formed_and_unknown_tools_defer():
    r = GrammarRung()
    r.add("convert", FX)
    assert r.check(ToolCall("convert", {"from_currency": "USD", "to_currency": "EUR"})).kind == VerdictKind.DEFER
    assert r.check(ToolCall("convert", {"named:from_currency": "USD", "to_currency": "EUR"})).kind == VerdictKind.DEFER
    assert r.check(ToolCall("other", {})).kind == VerdictKind.DEFER          # no grammar: fail-open


def test_alias_and_positional_repairs_and_misroute():
    r = GrammarRung()
    r.add("convert", FX)
    v = r.check(ToolCall("convert", {"from": "USD", "to": "EUR", "amount": 3}))
    assert v.kind == VerdictKind.TRANSFORM and v.reason == Reason.MISROUTE
    assert v.new_args == {"from_currency": "USD", "to_currency": "EUR", "amount": 3} and v.meta["repair"] == "alias"
    # an alias whose canonical key is already present is not renamed; the gap stays -> deny
    v = r.check(ToolCall("convert", {"from_currency": "USD", "from": "GBP"}))
    assert v.kind == VerdictKind.DENY and v.reason == Reason.MISROUTE and "to_currency" in v.claim
    v = r.check(ToolCall("convert", {"_positional": ["USD", "EUR", 10]}))
    assert v.kind == VerdictKind.TRANSFORM and v.new_args == {"from_currency": "USD", "to_currency": "EUR", "amount": 10}
    assert r.check(ToolCall("convert", {"_positional": ["USD"]})).kind == VerdictKind.DENY   # arity mismatch
    assert r.stats()["repairs"] == 2 and r.stats()["denies"] == 2


def test_grammars_dedupe_by_content_and_json_schema_order():
    r = GrammarRung()
    schema = {"properties": {"path": {"type": "string"}, "line": {"type": "integer"}}, "required": ["path"]}
    r.load_json_schema("Edit", schema)
    r.load_json_schema("Patch", dict(reversed(list(schema.items()))))
    r.register_openai_tools([{"type": "function", "function": {"name": "Read", "parameters": {
        "properties": {"path": {"type": "string"}}, "required": ["path"]}}}])
    assert r.has("Edit") and r.has("Read") and not r.has("Write")
    assert r.unique_grammars() == 2                                   # Edit and Patch share one entry
    assert [p.name for p in r.grammar("Edit").params] == ["line", "path"]
    assert r.check(ToolCall("Edit", {"line": 3})).kind == VerdictKind.DENY


def test_message_types_pack_validate_unpack():
    tr = TypeRegistry()
    a = tr.register("handoff", [Param("task", "string", True), Param("owner", "string", True), Param("note")])
    b = tr.register("handoff_v2", [Param("owner", "string", True), Param("task", "string", True), Param("note")])
    assert a.digest == b.digest and tr.unique_types() == 1
    assert tr.validate("handoff", {"task": "x"}) == (["owner"], True)
    assert tr.validate("nope", {}) == ([], False)
    assert tr.pack("handoff", {"task": "x"}) is None
    blob = tr.pack("handoff", {"task": "x", "owner": "a"})
    assert tr.unpack(blob) == ("handoff", {"task": "x", "owner": "a"})
    assert tr.unpack(blob.replace(a.digest.encode(), b"0" * 24)) is None   # digest must match the type
    assert tr.unpack(b"{not json") is None


def test_durability_promotion_fails_closed():
    assert all(known_durability(c) for c in ("turn", "session", "durable", "bounded"))
    assert not known_durability("eternal") and not known_durability("")
    v = may_promote("durable", PromotionMode.ENFORCE)
    assert v.promote and v.should_persist() and not v.would_refuse()
    for cls, reason in (("session", "non_durable"), ("bounded", "non_durable"), ("", "unknown_class")):
        w = may_promote(cls, PromotionMode.WARN)
        e = may_promote(cls, PromotionMode.ENFORCE)
        assert not w.promote and w.reason == reason and w.should_persist()     # warn: recorded, still persists
        assert not e.should_persist() and e.would_refuse()


def test_kernel_repairs_then_runs_the_policy_on_the_repaired_call():
    k = Kernel(policy_from_dict({"version": "fak-policy/v1", "allow": ["convert"]}))
    k.grammar.add("convert", FX)
    seen = []
    k.register("convert", lambda a: seen.append(a) or "ok")
    r = k.syscall(ToolCall("convert", {"from": "USD", "to": "EUR"}))
    assert r.status == Status.OK and seen == [{"from_currency": "USD", "to_currency": "EUR"}]
    assert r.verdict.kind == VerdictKind.TRANSFORM
    bad = k.syscall(ToolCall("convert", {"amount": 1}))
    assert bad.status == Status.ERROR and bad.verdict.reason == Reason.MISROUTE and not seen[1:]
    # a repaired call the policy refuses stays refused
    k2 = Kernel()
    k2.grammar.add("convert", FX)
    assert not k2.decide(ToolCall("convert", {"from": "USD", "to": "EUR"})).allowed
