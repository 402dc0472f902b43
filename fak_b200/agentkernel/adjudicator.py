"""The default-deny capability floor: every proposed tool call is adjudicated before it runs.

Rung order follows the reference monitor (internal/adjudicator/decide.go:317-640): provable
refusals first, then the affirmative allow, then the default-deny posture:

1. explicit policy deny (tool name -> reason);
2. SELF_MODIFY -- a write-shaped call whose target path hits a protected glob, and the shell
   form of the same (a write verb / redirect in a command string aimed at a protected path);
3. EGRESS_BLOCK -- a fetch-shaped call to a cloud-metadata / link-local / policy-denied host,
   or (with ``research_allow_hosts``) to any host outside the allowlist;
4. argument predicates (containment globs, deny regexes, size caps) -- restrict-only;
5. TRANSFORM -- secret-named argument fields are redacted before dispatch;
6. affirmative allow (exact name or prefix);
7. default deny, downgraded to admit-and-log for read-shaped tools under ADMIT_AND_LOG posture
   or for tools in the ``complain`` set.

Refusals carry a bounded witness (the offending glob / rule / host), never the policy itself
and never the argument value.
"""
from __future__ import annotations

import fnmatch
import ipaddress
import re
import threading
from urllib.parse import urlsplit

from .abi import Reason, ToolCall, Verdict, VerdictKind
from .policy import ArgKind, ArgPredicate, Policy, Posture, default_policy

_WRITE_WORDS = ("write", "edit", "create", "delete", "remove", "move", "rename", "patch", "put", "append", "mkdir",
                "notebookedit", "apply", "save", "upload")
_READ_WORDS = ("read", "get", "list", "search", "find", "lookup", "glob", "grep", "ls", "view", "fetch", "query",
               "describe", "show", "stat")
_PATH_KEYS = ("path", "file_path", "filepath", "filename", "target", "dest", "destination", "notebook_path", "dir")
_SHELL_TOOLS = ("bash", "shell", "sh", "exec", "run_command", "powershell", "terminal", "command")
_SHELL_WRITE = re.compile(r"(?:^|[\s;&|])(?:sed\s+-i|tee|cp|mv|rm|chmod|chown|truncate|install|ln|git\s+apply|"
                          r"git\s+checkout\s+--|dd)\b|>>?")
_FETCH_TOOLS = ("webfetch", "fetch", "http_get", "http_request", "curl", "download", "browse", "open_url")
_METADATA_HOSTS = {"169.254.169.254", "metadata.google.internal", "metadata", "fd00:ec2::254", "100.100.100.200"}


def write_shaped(tool: str) -> bool:
    t = tool.lower()
    return any(w in t for w in _WRITE_WORDS)


def read_shaped(tool: str) -> bool:
    t = tool.lower()
    return not write_shaped(tool) and any(t.startswith(w) or w in t for w in _READ_WORDS)


def _target_path(args: dict) -> str:
    for k in _PATH_KEYS:
        v = args.get(k)
        if isinstance(v, str) and v:
            return v
    return ""


def _glob_hit(path: str, globs: list[str]) -> str:
    p = path.replace("\\", "/")
    for g in globs:
        if g.endswith("/"):
            frag = g if g.startswith("/") else "/" + g
            if ("/" + p.lstrip("./") + "/").find(frag) >= 0 or p.startswith(g):
                return g
        elif any(ch in g for ch in "*?["):
            if fnmatch.fnmatch(p, g) or fnmatch.fnmatch(p.rsplit("/", 1)[-1], g):
                return g
        else:
            base = p.rsplit("/", 1)[-1]
            if base == g or base.startswith(g) or ("/" + g) in p or p == g:
                return g
    return ""


def _under_glob(glob: str, value: str) -> bool:
    """Containment: value is a path under glob's directory ("./out/**"); '..' escapes fail."""
    import posixpath
    root = glob.split("*", 1)[0].rstrip("/") or "."
    v = posixpath.normpath(value.replace("\\", "/"))
    r = posixpath.normpath(root)
    if v.startswith("../") or v == ".." or "/../" in v:
        return False
    return v == r or v.startswith(r.rstrip("/") + "/") or r == "."


def _host_blocked(host: str, extra: list[str]) -> bool:
    h = host.lower().strip("[]")
    if h in _METADATA_HOSTS or h in extra:
        return True
    try:
        ip = ipaddress.ip_address(h)
        return ip.is_link_local
    except ValueError:
        return False


class Adjudicator:
    def __init__(self, policy: Policy | None = None):
        self._lock = threading.RLock()
        self.set_policy(policy or default_policy())

    def set_policy(self, p: Policy) -> None:
        by_tool: dict[str, list[ArgPredicate]] = {}
        for ap in p.arg_predicates:
            by_tool.setdefault(ap.tool.lower(), []).append(ap)
        with self._lock:
            self.policy = p
            self._by_tool = by_tool

    # ---------------------------------------------------------------------------------
    def adjudicate(self, call: ToolCall) -> Verdict:
        with self._lock:
            p, preds = self.policy, self._by_tool.get(call.tool.lower(), [])
        args = call.args if isinstance(call.args, dict) else {}

        if call.tool in p.deny:
            return Verdict(VerdictKind.DENY, p.deny[call.tool], by="monitor", claim=call.tool)

        if write_shaped(call.tool):
            g = _glob_hit(_target_path(args), p.self_modify_globs)
            if g:
                return Verdict(VerdictKind.DENY, Reason.SELF_MODIFY, by="monitor", claim=g)
        if call.tool.lower() in _SHELL_TOOLS:
            cmd = args.get("command") or args.get("cmd") or ""
            if isinstance(cmd, str) and _SHELL_WRITE.search(cmd):
                for tok in re.split(r"[\s;&|<>'\"]+", cmd):
                    g = _glob_hit(tok, p.self_modify_globs) if tok else ""
                    if g:
                        return Verdict(VerdictKind.DENY, Reason.SELF_MODIFY, by="monitor", claim=g)

        if call.tool.lower() in _FETCH_TOOLS:
            url = args.get("url") or args.get("uri") or ""
            if isinstance(url, str) and url:
                host = urlsplit(url if "://" in url else "http://" + url).hostname or ""
                if _host_blocked(host, p.egress_deny_hosts):
                    return Verdict(VerdictKind.DENY, Reason.EGRESS_BLOCK, by="monitor", claim=host)
                if p.research_allow_hosts and not any(host == h or host.endswith("." + h)
                                                      for h in p.research_allow_hosts):
                    return Verdict(VerdictKind.DENY, Reason.POLICY_BLOCK, by="monitor", claim=host)

        advisory: list[str] = []
        for ap in preds:
            violated = False
            v = args.get(ap.arg)
            if ap.kind == ArgKind.ALLOW_GLOB:
                violated = not (isinstance(v, str) and _under_glob(ap.glob, v))
            elif ap.kind == ArgKind.DENY_REGEX:
                violated = isinstance(v, str) and ap.regex.search(v) is not None
            elif ap.kind == ArgKind.MAX_BYTES:
                violated = isinstance(v, str) and len(v.encode()) > ap.n
            if violated:
                claim = f"{ap.tool}.{ap.arg}:{ap.kind.name.lower()}"
                if ap.advisory:
                    advisory.append(claim)
                    continue
                return Verdict(VerdictKind.DENY, ap.reason, by="monitor", claim=claim)

        meta = {"advisory_violations": ",".join(advisory)} if advisory else {}
        allowed = call.tool in p.allow or any(call.tool.startswith(px) for px in p.allow_prefix)
        if allowed:
            red = {k: v for k, v in args.items() if k.lower() in p.redact_fields}
            if red:
                new = {k: ("[REDACTED]" if k.lower() in p.redact_fields else v) for k, v in args.items()}
                return Verdict(VerdictKind.TRANSFORM, Reason.NONE, by="monitor", new_args=new,
                               claim=",".join(sorted(red)), meta=meta)
            return Verdict(VerdictKind.ALLOW, Reason.NONE, by="monitor", meta=meta)

        if call.tool in p.complain or (p.posture == Posture.ADMIT_AND_LOG and read_shaped(call.tool)):
            meta = dict(meta, posture="admit_and_log", would_deny="DEFAULT_DENY")
            return Verdict(VerdictKind.ALLOW, Reason.NONE, by="monitor", meta=meta)
        return Verdict(VerdictKind.DENY, Reason.DEFAULT_DENY, by="monitor", claim=call.tool)

    def never_admits(self, tool: str) -> bool:
        p = self.policy
        if tool in p.deny:
            return True
        return not (tool in p.allow or any(tool.startswith(px) for px in p.allow_prefix) or tool in p.complain
                    or (p.posture == Posture.ADMIT_AND_LOG and read_shaped(tool)))
