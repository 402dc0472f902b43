"""Page pool and radix-tree prefix cache (pure-Python implementation).

``PagePool``: refcounted fixed-size KV pages (16 tokens each) -- the reference's
``PagedKVPool`` (internal/model/pagedkv.go:44-124).

``RadixCache``: a radix tree over token ids whose edges own whole KV pages, so a new
request that shares a prefix with any earlier one reuses those pages instead of
prefilling them again (reference ``radixkv.Tree``: Lookup internal/radixkv/radixkv.go:189,
Insert :211, split :149, LRU evictToBudget :252).  Differences by design:

* keys are matched in whole pages (16 tokens), because a page is the unit the attention
  kernels read through the block table;
* the tree stores page ids, not KV copies: a hit costs nothing but refcount bumps
  (the reference clones the matched KV into the new session, kv.go:14);
* eviction is LRU over leaves not referenced by any live sequence.

A C++ implementation with the same interface (``fak_b200._cpu.PagePool`` / ``RadixCache``,
csrc/cpu/radix.cpp) replaces these classes when the native extension is built (set
``FAK_PY_RADIX=1`` to keep the Python ones); this module is its executable specification.
"""
from __future__ import annotations

import os
import time


class OutOfPages(RuntimeError):
    """The KV page pool cannot satisfy an allocation even after evicting the cache."""


class PagePool:
    def __init__(self, n_pages: int, reserve: int = 1):
        # page 0..reserve-1 are never handed out (padding lanes of a CUDA graph point there)
        self.n_pages = n_pages
        self.reserve = reserve
        self.ref = [0] * n_pages
        self.free = list(range(n_pages - 1, reserve - 1, -1))

    def n_free(self) -> int:
        return len(self.free)

    def alloc(self, n: int) -> list[int]:
        if n > len(self.free):
            raise OutOfPages(f"need {n} KV pages, {len(self.free)} free")
        out = [self.free.pop() for _ in range(n)]
        for p in out:
            self.ref[p] = 1
        return out

    def retain(self, pages) -> None:
        for p in pages:
            if self.ref[p] <= 0:
                raise RuntimeError(f"retain of free page {p}")
            self.ref[p] += 1

    def release(self, pages) -> None:
        for p in pages:
            r = self.ref[p] - 1
            if r < 0:
                raise RuntimeError(f"double release of page {p}")
            self.ref[p] = r
            if r == 0:
                self.free.append(p)


class _Node:
    __slots__ = ("key", "pages", "children", "parent", "last_use")

    def __init__(self, key: tuple, pages: list[int], parent: "_Node | None"):
        self.key = key          # tokens on the edge into this node (multiple of page size)
        self.pages = pages      # one page per page_size tokens of key
        self.children: dict[tuple, _Node] = {}
        self.parent = parent
        self.last_use = time.monotonic()


class RadixCache:
    def __init__(self, pool: PagePool, page_size: int = 16):
        self.pool = pool
        self.ps = page_size
        self.root = _Node((), [], None)
        self.hits_tokens = 0
        self.lookup_tokens = 0
        self.n_cached_pages = 0

    # ------------------------------------------------------------------------------------
    def _chunk(self, tokens, i: int) -> tuple:
        return tuple(tokens[i:i + self.ps])

    def match(self, tokens) -> tuple[int, list[int], list[_Node]]:
        """Longest cached prefix in whole pages -> (n tokens, pages, path nodes)."""
        node, i, pages, path = self.root, 0, [], []
        n = len(tokens) - len(tokens) % self.ps
        while i < n:
            child = node.children.get(self._chunk(tokens, i))
            if child is None:
                break
            k = child.key
            m = 0
            while m < len(k) and i + m < n and k[m] == tokens[i + m]:
                m += 1
            m -= m % self.ps
            if m == 0:
                break
            if m < len(k):
                child = self._split(child, m)
            pages.extend(child.pages)
            path.append(child)
            i += m
            node = child
        now = time.monotonic()
        for nd in path:
            nd.last_use = now
        return i, pages, path

    def _split(self, node: _Node, m: int) -> _Node:
        """Split node's edge after m tokens; returns the new upper node."""
        parent = node.parent
        upper = _Node(node.key[:m], node.pages[: m // self.ps], parent)
        upper.last_use = node.last_use
        parent.children[self._chunk(node.key, 0)] = upper
        node.key = node.key[m:]
        node.pages = node.pages[m // self.ps:]
        node.parent = upper
        upper.children[self._chunk(node.key, 0)] = node
        return upper

    def lookup(self, tokens, max_tokens: int | None = None) -> tuple[int, list[int]]:
        """Match; the returned pages are retained for the caller (who releases them to the pool).

        A page referenced by a live sequence has refcount >= 2 (tree + sequence), which is
        what keeps it from being evicted.
        """
        limit = len(tokens) if max_tokens is None else min(len(tokens), max_tokens)
        n, pages, _ = self.match(list(tokens[:limit]))
        self.lookup_tokens += len(tokens)
        self.hits_tokens += n
        self.pool.retain(pages)
        return n, pages

    def insert(self, tokens, pages: list[int]) -> int:
        """Insert the whole-page prefix of ``tokens`` whose KV lives in ``pages``.

        The tree takes its own reference on every page it keeps.  Returns the number of
        tokens that were new to the tree.
        """
        n = min(len(tokens) - len(tokens) % self.ps, len(pages) * self.ps)
        node, i = self.root, 0
        added = 0
        while i < n:
            key = self._chunk(tokens, i)
            child = node.children.get(key)
            if child is None:
                new = _Node(tuple(tokens[i:n]), list(pages[i // self.ps: n // self.ps]), node)
                node.children[key] = new
                self.pool.retain(new.pages)
                self.n_cached_pages += len(new.pages)
                added += n - i
                break
            k = child.key
            m = 0
            while m < len(k) and i + m < n and k[m] == tokens[i + m]:
                m += 1
            m -= m % self.ps
            if m < len(k):
                child = self._split(child, m)
            child.last_use = time.monotonic()
            i += m
            node = child
        return added

    # ------------------------------------------------------------------------------------
    def _leaves(self):
        stack = [self.root]
        while stack:
            nd = stack.pop()
            if not nd.children and nd is not self.root:
                yield nd
            stack.extend(nd.children.values())

    def evict(self, n_pages: int) -> int:
        """Free up to n_pages by dropping least-recently-used unlocked leaves."""
        freed = 0
        while freed < n_pages:
            leaves = [nd for nd in self._leaves() if all(self.pool.ref[p] == 1 for p in nd.pages)]
            if not leaves:
                break
            victim = min(leaves, key=lambda nd: nd.last_use)
            parent = victim.parent
            del parent.children[self._chunk(victim.key, 0)]
            self.pool.release(victim.pages)
            self.n_cached_pages -= len(victim.pages)
            freed += len(victim.pages)
        return freed

    def sequences(self) -> list[tuple[list[int], list[int]]]:
        """(tokens, pages) of every root-to-leaf path -- what a session checkpoint saves."""
        out = []
        stack = [(self.root, [], [])]
        while stack:
            nd, toks, pages = stack.pop()
            toks, pages = toks + list(nd.key), pages + list(nd.pages)
            if not nd.children and nd is not self.root:
                out.append((toks, pages))
            for ch in nd.children.values():
                stack.append((ch, toks, pages))
        return sorted(out)

    def stats(self) -> dict:
        return {"cached_pages": self.n_cached_pages, "hit_tokens": self.hits_tokens,
                "lookup_tokens": self.lookup_tokens,
                "hit_rate": self.hits_tokens / self.lookup_tokens if self.lookup_tokens else 0.0}


# native implementation (same interface) when the C++ extension is built
PyPagePool, PyRadixCache = PagePool, RadixCache
if not os.environ.get("FAK_PY_RADIX"):
    try:
        import torch  # noqa: F401  (loads the libraries the extension links against)
        from .._cpu import PagePool, RadixCache  # noqa: F811
    except ImportError:
        pass
