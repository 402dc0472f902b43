"""Draft proposers for speculative decoding, and the acceptance walk of a speculation tree.

* ``LookupDrafter`` -- prompt lookup: find the longest recent n-gram (``max_n`` down to ``min_n``)
  that ends the context somewhere earlier in it (or in optional reference corpora) and propose the
  tokens that followed its most recent occurrence.  No model runs; it shines on agent transcripts
  that repeat tool output, code and JSON.
* ``MultiDrafter`` -- routes each round to one member drafter by its measured acceptance rate,
  after trying every member once and with a round-robin probe every ``probe_every`` rounds so a
  member whose luck changes is noticed.
* ``TreeLookupDrafter`` -- a speculation *tree*: the continuations after up to ``width`` distinct
  earlier occurrences of the context's suffix, merged into a trie (shared prefixes share nodes).
* ``accept_tree`` -- given each node's token and the target's greedy token at that node, the
  longest root-to-node path whose every token equals its parent's target token; the committed
  tokens are that path plus the target token at its end, which is exactly greedy decoding.

The engine verifies chains and trees with its own decode lanes (``engine.Engine`` spec paths);
these classes only propose and account.  Reference behaviour: internal/spec/drafters.go:42-330
(ModelDrafter, LookupDrafter, MultiDrafter) and the tree verify / AcceptTree of
internal/spec/verify.go:31-122 and internal/polymodel.
"""
from __future__ import annotations

import dataclasses

from .specmath import AcceptanceMeter


def _continuation(corpus: list[int], pat: list[int], limit: int, k: int, skip: int = 0) -> list[int] | None:
    """Tokens after the (skip + 1)-th most recent occurrence of ``pat`` starting before ``limit``."""
    n = len(pat)
    if n == 0 or n > len(corpus):
        return None
    limit = min(limit, len(corpus) - n)
    found = 0
    for i in range(limit - 1, -1, -1):
        if corpus[i:i + n] == pat:
            j = i + n
            if j >= len(corpus):
                continue
            if found == skip:
                return corpus[j:j + k]
            found += 1
    return None


class LookupDrafter:
    """Prompt lookup over the request's own context, with an incremental index: for every n in
    [min_n, max_n] the latest start of each n-gram that has a token after it, updated in O(max_n)
    per committed token (no rescans of a long agent transcript)."""

    def __init__(self, context: list[int], min_n: int = 1, max_n: int = 4, refs: list[list[int]] | None = None):
        self.min_n = max(1, min_n)
        self.max_n = max(self.min_n, min(8, max_n))
        self.refs = [list(r) for r in refs or []]
        self.seq: list[int] = []
        self.index: list[dict] = [dict() for _ in range(self.max_n + 1)]
        self.commit(context)

    HISTORY = 8   # starts remembered per n-gram (latest last)

    def commit(self, tokens: list[int]) -> None:
        for t in tokens:
            L = len(self.seq)            # the n-grams ending at L - 1 now have a follower (t)
            for n in range(self.min_n, self.max_n + 1):
                if L - n >= 0:
                    h = self.index[n].setdefault(tuple(self.seq[L - n:L]), [])
                    h.append(L - n)
                    if len(h) > self.HISTORY:
                        del h[0]
            self.seq.append(int(t))

    def starts(self, n: int) -> list[int]:
        """Earlier starts of the context's last n-gram that have a follower, latest first."""
        return list(reversed(self.index[n].get(tuple(self.seq[-n:]), [])))

    def draft(self, k: int) -> list[int]:
        if k <= 0 or not self.seq:
            return []
        for n in range(self.max_n, self.min_n - 1, -1):
            if n > len(self.seq):
                continue
            suf = tuple(self.seq[-n:])
            st = self.starts(n)
            if st:
                return self.seq[st[0] + n:st[0] + n + k]
            for ref in self.refs:
                c = _continuation(ref, list(suf), len(ref), k)
                if c:
                    return c
        return []


class MultiDrafter:
    def __init__(self, members: list[tuple[str, object]], probe_every: int = 8):
        self.members = members
        self.meters = [AcceptanceMeter() for _ in members]
        self.routed = [0] * len(members)
        self.probe_every = probe_every if probe_every > 0 else 8
        self.round = 0
        self._last: tuple[int, list[int]] | None = None

    def _pick(self) -> int:
        for i, n in enumerate(self.routed):
            if n == 0:
                return i
        if self.round % self.probe_every == self.probe_every - 1:
            return (self.round // self.probe_every) % len(self.members)
        return max(range(len(self.members)), key=lambda i: (self.meters[i].rate, -i))

    def draft(self, k: int) -> list[int]:
        i = self._pick()
        d = list(self.members[i][1].draft(k))[:max(0, k)]
        self._last = (i, d)
        self.routed[i] += 1
        self.round += 1
        return d

    def commit(self, tokens: list[int]) -> None:
        if self._last is not None:
            i, d = self._last
            acc = 0
            while acc < len(d) and acc < len(tokens) and d[acc] == tokens[acc]:
                acc += 1
            self.meters[i].observe(len(d), acc)
            self._last = None
        for _, m in self.members:
            m.commit(tokens)

    def stats(self) -> list[dict]:
        return [{"name": n, "rounds_routed": r, "drafted": m.drafted, "accepted": m.accepted, "rate": m.rate}
                for (n, _), r, m in zip(self.members, self.routed, self.meters)]


@dataclasses.dataclass
class SpecTree:
    """Non-root nodes in top-down order: ``tokens[i]`` with parent ``parent[i]`` (-1: the root, the
    current committed position)."""
    tokens: list[int]
    parent: list[int]

    def depth(self, i: int) -> int:
        d = 1
        p = self.parent[i]
        while p >= 0:
            d += 1
            p = self.parent[p]
        return d

    def leaves(self) -> list[int]:
        has_child = set(p for p in self.parent if p >= 0)
        return [i for i in range(len(self.tokens)) if i not in has_child]

    def path(self, i: int) -> list[int]:
        """Node indices root-side first, ending at i."""
        out = []
        while i >= 0:
            out.append(i)
            i = self.parent[i]
        return out[::-1]


class TreeLookupDrafter(LookupDrafter):
    def __init__(self, context: list[int], width: int = 3, min_n: int = 1, max_n: int = 4):
        super().__init__(context, min_n, max_n)
        self.width = max(1, width)

    def propose(self, depth: int) -> SpecTree:
        """Up to ``width`` continuations of length ``depth`` (distinct earlier occurrences of the
        longest matching suffix), merged into a trie."""
        conts: list[list[int]] = []
        for n in range(self.max_n, self.min_n - 1, -1):
            if n > len(self.seq):
                continue
            for i in self.starts(n):
                c = self.seq[i + n:i + n + depth]
                if c and c not in conts:
                    conts.append(c)
                if len(conts) >= self.width:
                    break
            if conts:
                break
        tokens: list[int] = []
        parent: list[int] = []
        children: dict[tuple[int, int], int] = {}
        # insert level by level so that every node comes after its parent
        for d in range(depth):
            for c in conts:
                if d >= len(c):
                    continue
                par = -1
                for j in range(d):
                    par = children[(par, c[j])]
                key = (par, c[d])
                if key not in children:
                    children[key] = len(tokens)
                    tokens.append(c[d])
                    parent.append(par)
        return SpecTree(tokens, parent)


def accept_tree(tree: SpecTree, root_target: int, node_target: list[int]) -> tuple[list[int], list[int]]:
    """(accepted node indices root-side first, committed tokens).  A child is accepted when its token
    equals its parent's target (greedy) token; among children the first in order wins.  The committed
    tokens are the accepted nodes' tokens plus the target token after the last one."""
    kids: dict[int, list[int]] = {}
    for i, p in enumerate(tree.parent):
        kids.setdefault(p, []).append(i)
    path: list[int] = []
    cur, want = -1, root_target
    while True:
        nxt = next((c for c in kids.get(cur, []) if tree.tokens[c] == want), None)
        if nxt is None:
            break
        path.append(nxt)
        cur, want = nxt, node_target[nxt]
    return path, [tree.tokens[i] for i in path] + [want]
