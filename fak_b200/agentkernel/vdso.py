"""Tool vDSO: answers a tool call locally, without running the tool, when that is provably the same
as running it.

Three tiers, consulted cheapest first:

1. pure registry -- tools declared pure (read-only and idempotent: the result is a function of the
   arguments alone) are computed in-process by their registered function;
2. content cache -- results of completed read-shaped calls keyed on (tool, sha256 of the canonical
   arguments, world version); any completed write-shaped call bumps the world version, so a read
   cached before a write is never served after it (a hit equals a fresh call);
3. static table -- canned answers for static tools (a version string, a capability list).

A hit still goes through adjudication first: the fast path only replaces execution.

Reference: internal/vdso/vdso.go (pure registry, content cache keyed on the world version, static
table; LRU capacity 1024).
"""
from __future__ import annotations

import collections
import hashlib
import json
import threading
from typing import Any, Callable

from .adjudicator import read_shaped, write_shaped

DEFAULT_CACHE_SIZE = 1024


def args_key(tool: str, args: dict) -> str:
    blob = json.dumps(args, sort_keys=True, separators=(",", ":"), default=str)
    return tool + ":" + hashlib.sha256(blob.encode()).hexdigest()


class VDSO:
    def __init__(self, cache_size: int = DEFAULT_CACHE_SIZE):
        self.pure: dict[str, Callable[[dict], Any]] = {}
        self.static: dict[str, Any] = {}
        self.cache: collections.OrderedDict[tuple[str, int], Any] = collections.OrderedDict()
        self.cache_size = cache_size
        self.world = 0
        self._lock = threading.Lock()
        self.stats = {"pure": 0, "cache": 0, "static": 0, "miss": 0, "world_bumps": 0}

    def register_pure(self, tool: str, fn: Callable[[dict], Any], read_only: bool = True,
                      idempotent: bool = True) -> None:
        """Only read-only, idempotent tools qualify (the hints are checked, not trusted blindly:
        a write-shaped tool name is refused)."""
        if not (read_only and idempotent) or write_shaped(tool):
            raise ValueError(f"vdso: {tool} is not pure (read-only and idempotent)")
        self.pure[tool] = fn

    def register_static(self, tool: str, answer: Any) -> None:
        self.static[tool] = answer

    def lookup(self, tool: str, args: dict) -> tuple[bool, Any, str]:
        """(hit, result, tier)."""
        if tool in self.pure:
            with self._lock:
                self.stats["pure"] += 1
            return True, self.pure[tool](args), "pure"
        key = (args_key(tool, args), self.world)
        with self._lock:
            if key in self.cache:
                self.cache.move_to_end(key)
                self.stats["cache"] += 1
                return True, self.cache[key], "cache"
            if tool in self.static:
                self.stats["static"] += 1
                return True, self.static[tool], "static"
            self.stats["miss"] += 1
        return False, None, ""

    def complete(self, tool: str, args: dict, result: Any, cacheable: bool = True) -> None:
        """Observe a completed call: writes (and calls of unknown shape) advance the world, reads
        fill the cache with ``result`` -- the content the model was shown."""
        with self._lock:
            if write_shaped(tool) or not read_shaped(tool):
                self.world += 1
                self.stats["world_bumps"] += 1
                self.cache.clear()   # every entry belongs to an older world now
                return
            if not cacheable:
                return
            self.cache[(args_key(tool, args), self.world)] = result
            self.cache.move_to_end((args_key(tool, args), self.world))
            while len(self.cache) > self.cache_size:
                self.cache.popitem(last=False)
