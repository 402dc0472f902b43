"""Decode constraints: logit bias and token masks applied at the token-selection boundary.

A ``LogitMask`` sets disallowed tokens to -inf before any bias, so a mask is a hard structural
constraint and a bias a soft preference (a masked token stays masked whatever its bias).  Masks are
dormant unless guided decoding is switched on (``FAK_NATIVE_GUIDED_DECODE=1``), so a compiled-in
mask never changes a default decode; an empty bias and a dormant mask leave greedy decoding exactly
the argmax path.

Masks:

* ``AllowedSetMask`` -- the same allowed token set at every step (e.g. one of the tool names);
* ``StepMask`` -- a different allowed set per generated token; steps past the list are free;
* ``JsonMask`` -- only tokens whose text keeps the output a prefix of a valid JSON value (a
  character-level pushdown automaton walked over a trie of the vocabulary's token strings).

Reference: DecodeConstraint / LogitMask / AllowedSetMask / StepMask and the guided-decode flag
(internal/model/constraint.go:60-201); logit-bias clamp (internal/agent/inkernel_sampling.go).
"""
from __future__ import annotations

import os
import re

import torch

LOGIT_BIAS_CLAMP = 100.0


def guided_decode_enabled() -> bool:
    return os.environ.get("FAK_NATIVE_GUIDED_DECODE") == "1"


class LogitMask:
    def allowed(self, history: list[int], vocab_size: int) -> torch.Tensor | None:
        """Bool tensor [vocab_size] of allowed tokens, or None for "everything allowed"."""
        raise NotImplementedError

    def apply(self, history: list[int], logits: torch.Tensor) -> torch.Tensor:
        ok = self.allowed(history, logits.numel())
        if ok is None:
            return logits
        return logits.masked_fill(~ok.to(logits.device), float("-inf"))


class AllowedSetMask(LogitMask):
    def __init__(self, tokens):
        self.tokens = sorted(set(int(t) for t in tokens))

    def allowed(self, history, vocab_size):
        ok = torch.zeros(vocab_size, dtype=torch.bool)
        idx = [t for t in self.tokens if 0 <= t < vocab_size]
        if idx:
            ok[torch.tensor(idx)] = True
        return ok


class StepMask(LogitMask):
    def __init__(self, per_step):
        self.per_step = [None if s is None else AllowedSetMask(s) for s in per_step]

    def allowed(self, history, vocab_size):
        k = len(history)
        if k >= len(self.per_step) or self.per_step[k] is None:
            return None
        return self.per_step[k].allowed(history, vocab_size)


# ---- JSON prefix automaton -------------------------------------------------------------------
_WS = " \t\n\r"
_NUM_PREFIX = re.compile(r"-?|-?(0|[1-9]\d*)(\.\d+)?([eE][+-]?\d*)?|-?(0|[1-9]\d*)\.")
_NUM_FULL = re.compile(r"-?(0|[1-9]\d*)(\.\d+)?([eE][+-]?\d+)?")


class _Json:
    """Character-level recogniser of prefixes of one JSON value.  ``feed`` returns False when the
    character cannot continue a valid JSON text; ``done`` turns True once the top-level value is
    complete (only whitespace may follow).  Frames: ("o", phase) with phase in key_or_end / key /
    colon / value / comma_or_end, ("a", phase) with phase in value_or_end / value / comma_or_end."""

    __slots__ = ("stack", "mode", "text", "esc", "uni", "is_key", "done")

    def __init__(self):
        self.stack: list[list[str]] = []
        self.mode = "ws"      # ws | str | num | lit
        self.text = ""        # number so far / literal remainder
        self.esc = False
        self.uni = 0
        self.is_key = False
        self.done = False

    def copy(self) -> "_Json":
        c = _Json.__new__(_Json)
        c.stack = [list(f) for f in self.stack]
        c.mode, c.text, c.esc, c.uni, c.is_key, c.done = (self.mode, self.text, self.esc, self.uni, self.is_key,
                                                          self.done)
        return c

    def _complete(self) -> None:
        self.mode = "ws"
        if not self.stack:
            self.done = True
            return
        f = self.stack[-1]
        f[1] = "comma_or_end"

    def _start_value(self, ch: str) -> bool:
        if ch == "{":
            self.stack.append(["o", "key_or_end"])
        elif ch == "[":
            self.stack.append(["a", "value_or_end"])
        elif ch == '"':
            self.mode, self.is_key = "str", False
        elif ch == "-" or ch.isdigit():
            self.mode, self.text = "num", ch
        elif ch in "tfn":
            self.mode, self.text = "lit", {"t": "rue", "f": "alse", "n": "ull"}[ch]
        else:
            return False
        return True

    def feed(self, ch: str) -> bool:
        if self.mode == "str":
            if self.uni:
                if ch not in "0123456789abcdefABCDEF":
                    return False
                self.uni -= 1
            elif self.esc:
                if ch == "u":
                    self.uni = 4
                elif ch not in '"\\/bfnrt':
                    return False
                self.esc = False
            elif ch == "\\":
                self.esc = True
            elif ch == '"':
                if self.is_key:
                    self.mode = "ws"
                    self.stack[-1][1] = "colon"
                else:
                    self._complete()
            elif ord(ch) < 0x20:
                return False
            return True
        if self.mode == "lit":
            if ch != self.text[0]:
                return False
            self.text = self.text[1:]
            if not self.text:
                self._complete()
            return True
        if self.mode == "num":
            if _NUM_PREFIX.fullmatch(self.text + ch):
                self.text += ch
                return True
            if not _NUM_FULL.fullmatch(self.text):
                return False
            self._complete()
        if ch in _WS:
            return True
        if self.done:
            return False
        if not self.stack:
            return self._start_value(ch)
        kind, phase = self.stack[-1]
        if kind == "o":
            if phase in ("key_or_end", "key") and ch == '"':
                self.mode, self.is_key = "str", True
                return True
            if phase == "key_or_end" and ch == "}" or phase == "comma_or_end" and ch == "}":
                self.stack.pop()
                self._complete()
                return True
            if phase == "colon" and ch == ":":
                self.stack[-1][1] = "value"
                return True
            if phase == "comma_or_end" and ch == ",":
                self.stack[-1][1] = "key"
                return True
            if phase == "value":
                return self._start_value(ch)
            return False
        if phase in ("value_or_end", "comma_or_end") and ch == "]":
            self.stack.pop()
            self._complete()
            return True
        if phase == "comma_or_end" and ch == ",":
            self.stack[-1][1] = "value"
            return True
        if phase in ("value_or_end", "value"):
            return self._start_value(ch)
        return False

    def complete(self) -> bool:
        """True when the text so far is a whole JSON value (a trailing number counts)."""
        if self.done:
            return True
        return self.mode == "num" and not self.stack and bool(_NUM_FULL.fullmatch(self.text))


class JsonMask(LogitMask):
    """Allows the tokens whose text keeps the generated text a prefix of one JSON value, and EOS
    once the value is complete.  ``token_text(id)`` gives a token's decoded text."""

    def __init__(self, token_text, vocab_size: int, eos_id: int | None = None):
        self.vocab_size = vocab_size
        self.eos_id = eos_id
        self.trie: dict = {}
        self.text = {}
        for t in range(vocab_size):
            s = token_text(t)
            if not s:
                continue
            self.text[t] = s
            node = self.trie
            for ch in s:
                node = node.setdefault(ch, {})
            node.setdefault(None, []).append(t)

    def _state(self, history: list[int]) -> _Json | None:
        st = _Json()
        for t in history:
            for ch in self.text.get(t, ""):
                if not st.feed(ch):
                    return None
        return st

    def allowed(self, history, vocab_size):
        ok = torch.zeros(vocab_size, dtype=torch.bool)
        st = self._state(history)
        if st is None:
            return ok
        if st.complete() and self.eos_id is not None and 0 <= self.eos_id < vocab_size:
            ok[self.eos_id] = True
        out: list[int] = []
        stack = [(self.trie, st)]
        while stack:
            node, s = stack.pop()
            for ch, child in node.items():
                if ch is None:
                    out.extend(child)
                    continue
                s2 = s.copy()
                if s2.feed(ch):
                    stack.append((child, s2))
        if out:
            ok[torch.tensor([t for t in out if t < vocab_size], dtype=torch.long)] = True
        return ok


def apply_constraint(row: torch.Tensor, mask: LogitMask | None, bias: dict[int, float] | None,
                     history: list[int]) -> torch.Tensor:
    """Mask first (hard), then clamped logit bias (soft); out-of-vocabulary bias entries are ignored."""
    if mask is not None and guided_decode_enabled():
        row = mask.apply(history, row)
    if bias:
        V = row.numel()
        items = [(t, max(-LOGIT_BIAS_CLAMP, min(LOGIT_BIAS_CLAMP, float(b)))) for t, b in bias.items() if 0 <= t < V]
        if items:
            row = row.clone()
            row[torch.tensor([t for t, _ in items], device=row.device)] += torch.tensor(
                [b for _, b in items], device=row.device, dtype=row.dtype)
    return row
