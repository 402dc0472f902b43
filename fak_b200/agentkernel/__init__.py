"""Agent-kernel security spine: syscall ABI, default-deny adjudicator, result admission, journal."""
from .abi import Reason, Result, Status, ToolCall, Verdict, VerdictKind
from .adjudicator import Adjudicator
from .ctxmmu import ContextMMU
from .journal import Journal
from .kernel import Kernel
from .policy import Policy, PolicyError, Posture, default_policy, load_policy, policy_from_dict

__all__ = ["Reason", "Result", "Status", "ToolCall", "Verdict", "VerdictKind", "Adjudicator", "ContextMMU", "Journal",
           "Kernel", "Policy", "PolicyError", "Posture", "default_policy", "load_policy", "policy_from_dict"]
