"""Byte-level BPE tokenizer built from a GGUF vocabulary or a HF tokenizer.json.

Behaviour follows the reference's tokenizer leaf (internal/tokenizer/tokenizer.go:33-290,
ggml.go:38): merge ranks, added/special tokens matched before pre-tokenization,
a pre-tokenizer chosen per family (GPT-2/SmolLM2 ByteLevel regex vs the
Qwen2 Split regex), and a ByteLevel decoder.  ``IncrementalDecoder`` yields text
only once a UTF-8 sequence is complete (reference: incremental.go:11-100).
"""
from __future__ import annotations

import functools
import json
from typing import Iterable

import regex

GPT2_PATTERN = r"""'s|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+"""
QWEN2_PATTERN = (r"""(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}| ?[^\s\p{L}\p{N}]+[\r\n]*"""
                 r"""|\s*[\r\n]+|\s+(?!\S)|\s+""")


@functools.lru_cache(maxsize=1)
def bytes_to_unicode() -> dict[int, str]:
    """GPT-2's reversible byte -> printable unicode map."""
    bs = list(range(ord("!"), ord("~") + 1)) + list(range(ord("¡"), ord("¬") + 1)) + list(range(ord("®"), ord("ÿ") + 1))
    cs = bs[:]
    n = 0
    for b in range(256):
        if b not in bs:
            bs.append(b)
            cs.append(256 + n)
            n += 1
    return {b: chr(c) for b, c in zip(bs, cs)}


class Tokenizer:
    def __init__(self, tokens: list[str], merges: Iterable[str], special_ids: Iterable[int] = (),
                 pattern: str = GPT2_PATTERN, bos_id: int | None = None, eos_id: int | None = None):
        self.id_to_token = list(tokens)
        self.token_to_id = {t: i for i, t in enumerate(self.id_to_token)}
        self.merge_rank: dict[tuple[str, str], int] = {}
        for r, m in enumerate(merges):
            parts = m.split(" ")
            if len(parts) == 2:
                self.merge_rank.setdefault((parts[0], parts[1]), r)
        self.special = {i: self.id_to_token[i] for i in special_ids}
        specials_sorted = sorted(self.special.items(), key=lambda kv: -len(kv[1]))
        self._special_re = (regex.compile("|".join(regex.escape(s) for _, s in specials_sorted))
                            if specials_sorted else None)
        self._special_by_text = {s: i for i, s in self.special.items()}
        self._pat = regex.compile(pattern)
        self._b2u = bytes_to_unicode()
        self._u2b = {v: k for k, v in self._b2u.items()}
        self.bos_id = bos_id
        self.eos_id = eos_id
        self._cache: dict[str, list[int]] = {}

    # ---------------------------------------------------------------------------------
    @classmethod
    def from_gguf_metadata(cls, meta: dict) -> "Tokenizer":
        model = meta.get("tokenizer.ggml.model", "gpt2")
        if model != "gpt2":
            raise NotImplementedError(f"tokenizer model {model!r} (only byte-level BPE 'gpt2' is supported)")
        tokens = meta["tokenizer.ggml.tokens"]
        types = meta.get("tokenizer.ggml.token_type", [1] * len(tokens))
        merges = meta.get("tokenizer.ggml.merges", [])
        pre = meta.get("tokenizer.ggml.pre", "")
        arch = meta.get("general.architecture", "")
        pattern = QWEN2_PATTERN if (pre.startswith("qwen") or arch.startswith("qwen")) else GPT2_PATTERN
        special = [i for i, t in enumerate(types) if t in (3, 4)]
        return cls(tokens, merges, special, pattern, meta.get("tokenizer.ggml.bos_token_id"),
                   meta.get("tokenizer.ggml.eos_token_id"))

    @classmethod
    def from_tokenizer_json(cls, path: str) -> "Tokenizer":
        with open(path, encoding="utf-8") as f:
            tj = json.load(f)
        model = tj["model"]
        if model.get("type") != "BPE":
            raise NotImplementedError("only BPE tokenizer.json is supported")
        vocab = model["vocab"]
        added = {a["id"]: a["content"] for a in tj.get("added_tokens", [])}
        n = max(list(vocab.values()) + list(added) + [-1]) + 1
        tokens = [f"<|unused_{i}|>" for i in range(n)]
        for t, i in vocab.items():
            tokens[i] = t
        for i, t in added.items():
            tokens[i] = t
        merges = [m if isinstance(m, str) else " ".join(m) for m in model.get("merges", [])]
        pre = json.dumps(tj.get("pre_tokenizer") or {})
        pattern = QWEN2_PATTERN if "Split" in pre and "\\p{N}" in pre else GPT2_PATTERN
        special = [a["id"] for a in tj.get("added_tokens", []) if a.get("special", True)]
        return cls(tokens, merges, special, pattern)

    # ---------------------------------------------------------------------------------
    @property
    def vocab_size(self) -> int:
        return len(self.id_to_token)

    def _bpe(self, word: str) -> list[int]:
        hit = self._cache.get(word)
        if hit is not None:
            return hit
        parts = list(word)
        rank = self.merge_rank
        while len(parts) > 1:
            best, best_i = None, -1
            for i in range(len(parts) - 1):
                r = rank.get((parts[i], parts[i + 1]))
                if r is not None and (best is None or r < best):
                    best, best_i = r, i
            if best is None:
                break
            parts[best_i:best_i + 2] = [parts[best_i] + parts[best_i + 1]]
        ids = []
        for p in parts:
            i = self.token_to_id.get(p)
            if i is None:  # not in vocab: fall back to single byte-symbols
                ids.extend(self.token_to_id[c] for c in p)
            else:
                ids.append(i)
        if len(self._cache) < 65536:
            self._cache[word] = ids
        return ids

    def _encode_plain(self, text: str, out: list[int]) -> None:
        for piece in self._pat.findall(text):
            mapped = "".join(self._b2u[b] for b in piece.encode("utf-8"))
            out.extend(self._bpe(mapped))

    def encode(self, text: str, allow_special: bool = True) -> list[int]:
        out: list[int] = []
        if allow_special and self._special_re is not None:
            pos = 0
            for m in self._special_re.finditer(text):
                if m.start() > pos:
                    self._encode_plain(text[pos:m.start()], out)
                out.append(self._special_by_text[m.group(0)])
                pos = m.end()
            if pos < len(text):
                self._encode_plain(text[pos:], out)
        else:
            self._encode_plain(text, out)
        return out

    def token_bytes(self, i: int) -> bytes:
        t = self.id_to_token[i]
        if i in self.special:
            return t.encode("utf-8")
        try:
            return bytes(self._u2b[c] for c in t)
        except KeyError:
            return t.encode("utf-8")

    def decode(self, ids: Iterable[int], skip_special: bool = False) -> str:
        buf = bytearray()
        for i in ids:
            if skip_special and i in self.special:
                continue
            buf += self.token_bytes(int(i))
        return buf.decode("utf-8", errors="replace")


class IncrementalDecoder:
    """Streams text for generated ids, holding back incomplete UTF-8 sequences."""

    def __init__(self, tok: Tokenizer, skip_special: bool = True):
        self.tok = tok
        self.skip_special = skip_special
        self._pending = bytearray()

    def push(self, token_id: int) -> str:
        if self.skip_special and token_id in self.tok.special:
            return ""
        self._pending += self.tok.token_bytes(token_id)
        # emit the longest prefix that is complete UTF-8
        for cut in range(len(self._pending), max(len(self._pending) - 4, -1), -1):
            try:
                s = self._pending[:cut].decode("utf-8")
            except UnicodeDecodeError:
                continue
            del self._pending[:cut]
            return s
        return ""

    def flush(self) -> str:
        s = self._pending.decode("utf-8", errors="replace")
        self._pending.clear()
        return s
