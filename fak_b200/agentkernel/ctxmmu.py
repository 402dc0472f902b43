"""Result admission ("context MMU"): screen tool results before they enter the model context.

Results that carry credentials are quarantined or redacted (reference: internal/ctxmmu/mmu.go,
the on-discovery secret rung internal/secretgate), oversize results are truncated to the
context budget, and prompt-injection markers are fenced as untrusted data.
"""
from __future__ import annotations

import dataclasses
import re

from .abi import Reason, Verdict, VerdictKind

SECRET_PATTERNS = [
    re.compile(r"AKIA[0-9A-Z]{16}"),                                  # AWS access key id
    re.compile(r"-----BEGIN (?:RSA |EC |OPENSSH |DSA |PGP )?PRIVATE KEY-----"),
    re.compile(r"\bgh[pousr]_[A-Za-z0-9]{36,}\b"),                     # GitHub tokens
    re.compile(r"\bsk-[A-Za-z0-9_-]{20,}\b"),                          # API secret keys
    re.compile(r"\bxox[abposr]-[A-Za-z0-9-]{10,}\b"),                  # Slack tokens
    re.compile(r"\bAIza[0-9A-Za-z_-]{35}\b"),                          # Google API keys
    re.compile(r"(?i)\b(?:password|passwd|secret|api[_-]?key)\s*[:=]\s*['\"]?[^\s'\"]{8,}"),
]
INJECTION_MARKERS = [
    re.compile(r"(?i)ignore (?:all |any )?(?:previous|prior) instructions"),
    re.compile(r"(?i)<\|im_start\|>\s*system"),
    re.compile(r"(?i)you are now (?:in )?developer mode"),
]


@dataclasses.dataclass
class Admission:
    verdict: Verdict
    content: str
    findings: list[str]


class ContextMMU:
    def __init__(self, budget_chars: int = 200_000, posture: str = "quarantine", extra_patterns=()):
        if posture not in ("quarantine", "fail_closed", "admit_and_log"):
            raise ValueError("posture must be quarantine, fail_closed or admit_and_log")
        self.budget = budget_chars
        self.posture = posture
        self.patterns = list(SECRET_PATTERNS) + list(extra_patterns)

    def admit(self, tool: str, content: str) -> Admission:
        text = content if isinstance(content, str) else str(content)
        findings = []
        for pat in self.patterns:
            if pat.search(text):
                findings.append(pat.pattern[:32])
        if findings:
            if self.posture == "fail_closed":
                return Admission(Verdict(VerdictKind.DENY, Reason.RESULT_SECRET_DISCOVERED, by="ctxmmu",
                                         claim=f"{len(findings)} secret pattern(s)"), "", findings)
            redacted = text
            for pat in self.patterns:
                redacted = pat.sub("[REDACTED-SECRET]", redacted)
            if self.posture == "quarantine":
                return Admission(Verdict(VerdictKind.QUARANTINE, Reason.RESULT_SECRET_DISCOVERED, by="ctxmmu",
                                         claim=f"{len(findings)} secret pattern(s)"), redacted, findings)
            return Admission(Verdict(VerdictKind.ALLOW, Reason.NONE, by="ctxmmu",
                                     meta={"posture": "admit_and_log", "would_deny": "RESULT_SECRET_DISCOVERED"}),
                             text, findings)
        if any(m.search(text) for m in INJECTION_MARKERS):
            text = "<untrusted-tool-output>\n" + text + "\n</untrusted-tool-output>"
            findings.append("injection-marker")
        if len(text) > self.budget:
            text = text[: self.budget] + f"\n[... truncated {len(text) - self.budget} chars]"
            return Admission(Verdict(VerdictKind.TRANSFORM, Reason.OVERSIZE, by="ctxmmu"), text, findings)
        return Admission(Verdict(VerdictKind.ALLOW, Reason.NONE, by="ctxmmu"), text, findings)
