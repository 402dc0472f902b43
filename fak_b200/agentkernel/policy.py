"""Policy manifests for the capability floor.

A policy is JSON (``"version": "fak-policy/v1"``) with the same keys as the reference's
manifests (internal/policy, cmd/fak/guard-default-policy.json): ``allow``, ``allow_prefix``,
``deny`` (tool -> reason), ``arg_rules`` (per-tool argument predicates), ``self_modify_globs``,
``redact_fields``, ``posture``, ``complain``, ``egress`` (``deny_hosts``), ``research_allow_hosts``.
Validation is fail-loud at load: an unknown key, a bad regex or an unknown reason name is an
error, never a silently weaker floor.
"""
from __future__ import annotations

import dataclasses
import enum
import json
import re
from typing import Any

from .abi import Reason


class Posture(enum.IntEnum):
    FAIL_CLOSED = 0     # anything not affirmatively allowed is denied
    ADMIT_AND_LOG = 1   # low-risk read-shaped default-denies are admitted with a would-deny record


class ArgKind(enum.IntEnum):
    ALLOW_GLOB = 1      # the arg must be a path under the glob (a missing arg violates)
    DENY_REGEX = 2      # an arg matching the regex is denied
    MAX_BYTES = 3       # a string arg longer than N bytes is denied


@dataclasses.dataclass
class ArgPredicate:
    tool: str
    arg: str
    kind: ArgKind
    glob: str = ""
    regex: re.Pattern | None = None
    n: int = 0
    reason: Reason = Reason.POLICY_BLOCK
    advisory: bool = False


@dataclasses.dataclass
class Policy:
    posture: Posture = Posture.FAIL_CLOSED
    allow: set[str] = dataclasses.field(default_factory=set)
    allow_prefix: list[str] = dataclasses.field(default_factory=list)
    deny: dict[str, Reason] = dataclasses.field(default_factory=dict)
    self_modify_globs: list[str] = dataclasses.field(default_factory=list)
    redact_fields: list[str] = dataclasses.field(default_factory=list)
    arg_predicates: list[ArgPredicate] = dataclasses.field(default_factory=list)
    complain: set[str] = dataclasses.field(default_factory=set)
    egress_deny_hosts: list[str] = dataclasses.field(default_factory=list)
    research_allow_hosts: list[str] = dataclasses.field(default_factory=list)
    secret_patterns: list[re.Pattern] = dataclasses.field(default_factory=list)
    version: str = "fak-policy/v1"


_KEYS = {"version", "allow", "allow_prefix", "deny", "arg_rules", "self_modify_globs", "redact_fields", "posture",
         "complain", "egress", "research_allow_hosts", "secret_patterns", "comment", "description"}


class PolicyError(ValueError):
    pass


def policy_from_dict(d: dict[str, Any]) -> Policy:
    unknown = set(d) - _KEYS
    if unknown:
        raise PolicyError(f"unknown policy keys: {sorted(unknown)}")
    if d.get("version", "fak-policy/v1") != "fak-policy/v1":
        raise PolicyError(f"unsupported policy version {d.get('version')!r}")
    p = Policy()
    posture = str(d.get("posture", "fail_closed")).lower()
    if posture not in ("fail_closed", "admit_and_log"):
        raise PolicyError(f"posture must be fail_closed or admit_and_log, not {posture!r}")
    p.posture = Posture.FAIL_CLOSED if posture == "fail_closed" else Posture.ADMIT_AND_LOG
    p.allow = set(d.get("allow", []))
    p.allow_prefix = list(d.get("allow_prefix", []))
    try:
        p.deny = {k: Reason.parse(v) for k, v in dict(d.get("deny", {})).items()}
    except KeyError as e:
        raise PolicyError(f"unknown reason in deny: {e}") from e
    p.self_modify_globs = list(d.get("self_modify_globs", []))
    p.redact_fields = [f.lower() for f in d.get("redact_fields", [])]
    p.complain = set(d.get("complain", []))
    egress = d.get("egress", {}) or {}
    p.egress_deny_hosts = [h.lower() for h in egress.get("deny_hosts", [])]
    p.research_allow_hosts = [h.lower() for h in d.get("research_allow_hosts", [])]
    for pat in d.get("secret_patterns", []):
        try:
            p.secret_patterns.append(re.compile(pat))
        except re.error as e:
            raise PolicyError(f"bad secret pattern {pat!r}: {e}") from e
    for i, r in enumerate(d.get("arg_rules", [])):
        kinds = [k for k in ("allow_glob", "deny_regex", "max_bytes") if k in r]
        if len(kinds) != 1:
            raise PolicyError(f"arg_rules[{i}]: exactly one of allow_glob/deny_regex/max_bytes required")
        if not r.get("tool") or not r.get("arg"):
            raise PolicyError(f"arg_rules[{i}]: tool and arg are required")
        try:
            reason = Reason.parse(r.get("reason", "POLICY_BLOCK"))
        except KeyError as e:
            raise PolicyError(f"arg_rules[{i}]: unknown reason {r.get('reason')!r}") from e
        k = kinds[0]
        ap = ArgPredicate(tool=r["tool"], arg=r["arg"], kind=ArgKind[k.upper()], reason=reason,
                          advisory=bool(r.get("advisory", False)))
        if k == "allow_glob":
            ap.glob = r[k]
        elif k == "deny_regex":
            try:
                ap.regex = re.compile(r[k])
            except re.error as e:
                raise PolicyError(f"arg_rules[{i}]: bad regex: {e}") from e
        else:
            ap.n = int(r[k])
            if ap.n <= 0:
                raise PolicyError(f"arg_rules[{i}]: max_bytes must be positive")
        p.arg_predicates.append(ap)
    return p


def load_policy(path: str) -> Policy:
    with open(path, encoding="utf-8") as f:
        return policy_from_dict(json.load(f))


def default_policy() -> Policy:
    """The built-in floor for wrapped coding agents: allow the common agent tools, refuse the
    destructive shell shapes, protect credentials and VCS metadata, redact secret fields."""
    return policy_from_dict({
        "version": "fak-policy/v1",
        "allow": ["Bash", "BashOutput", "KillShell", "Read", "Edit", "Write", "NotebookEdit", "Glob", "Grep", "LS",
                  "TodoWrite", "Task", "WebFetch", "WebSearch", "ExitPlanMode", "Skill", "SlashCommand", "Agent",
                  "AskUserQuestion", "TaskCreate", "TaskGet", "TaskList", "TaskOutput", "TaskStop", "TaskUpdate",
                  "ToolSearch"],
        "allow_prefix": ["read_", "get_", "search_", "list_", "lookup_", "find_"],
        "arg_rules": [
            {"tool": "Bash", "arg": "command", "deny_regex": r"\brm\s+-[A-Za-z]*[rRfF]", "reason": "POLICY_BLOCK"},
            {"tool": "Bash", "arg": "command", "deny_regex": r"\bsudo\b", "reason": "POLICY_BLOCK"},
            {"tool": "Bash", "arg": "command", "deny_regex": r"\bmkfs\b|\bdd\s+if=|>\s*/dev/sd", "reason": "POLICY_BLOCK"},
            {"tool": "Bash", "arg": "command", "deny_regex": r":\(\)\s*\{", "reason": "POLICY_BLOCK"},
            {"tool": "Bash", "arg": "command", "deny_regex": r"\b(curl|wget)\b[^|]*\|\s*(sudo\s+)?(ba)?sh\b",
             "reason": "POLICY_BLOCK"},
        ],
        "self_modify_globs": [".git/", ".env", ".aws/", ".npmrc", ".netrc", "id_rsa", "id_ed25519", "/etc/"],
        "redact_fields": ["password", "secret", "api_key", "token", "authorization"],
    })
