"""Hash-chained audit journal of kernel decisions.

Each entry is one JSON line carrying the SHA-256 of the previous line, so any edit, deletion or
reordering breaks ``verify()``.  Arguments are recorded as a digest plus their key names, never
their values (the reference's decision journal records the same bounded facts:
internal/journal, cmd/fak/guard.go:116).
"""
from __future__ import annotations

import hashlib
import json
import os
import threading
import time
from typing import Iterator

GENESIS = "0" * 64


def _digest(obj) -> str:
    return hashlib.sha256(json.dumps(obj, sort_keys=True, default=str).encode()).hexdigest()


class Journal:
    def __init__(self, path: str | None = None):
        self.path = path
        self._lock = threading.Lock()
        self._entries: list[dict] = []
        self.head = GENESIS
        if path and os.path.exists(path):
            for e in self.read(path):
                self._entries.append(e)
                self.head = e["hash"]

    def append(self, kind: str, **fields) -> dict:
        with self._lock:
            e = {"seq": len(self._entries), "ts": time.time(), "kind": kind, "prev": self.head, **fields}
            e["hash"] = hashlib.sha256((self.head + json.dumps(e, sort_keys=True, default=str)).encode()).hexdigest()
            self._entries.append(e)
            self.head = e["hash"]
            if self.path:
                with open(self.path, "a", encoding="utf-8") as f:
                    f.write(json.dumps(e, sort_keys=True, default=str) + "\n")
            return e

    def record_decision(self, call, verdict) -> dict:
        return self.append("decision", tool=call.tool, seq=call.seq, trace_id=call.trace_id,
                           arg_keys=sorted(call.args) if isinstance(call.args, dict) else [],
                           args_digest=_digest(call.args), verdict=verdict.to_dict())

    def entries(self) -> list[dict]:
        with self._lock:
            return list(self._entries)

    @staticmethod
    def read(path: str) -> Iterator[dict]:
        with open(path, encoding="utf-8") as f:
            for line in f:
                line = line.strip()
                if line:
                    yield json.loads(line)

    @staticmethod
    def verify_entries(entries: list[dict]) -> tuple[bool, int]:
        """(ok, index of the first bad entry or -1)."""
        prev = GENESIS
        for i, e in enumerate(entries):
            body = {k: v for k, v in e.items() if k != "hash"}
            if body.get("prev") != prev:
                return False, i
            h = hashlib.sha256((prev + json.dumps(body, sort_keys=True, default=str)).encode()).hexdigest()
            if h != e.get("hash"):
                return False, i
            prev = h
        return True, -1

    def verify(self) -> tuple[bool, int]:
        return self.verify_entries(self.entries())
