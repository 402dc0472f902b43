"""Speculative-decoding drafters and the tree acceptance walk (CPU)."""
from fak_b200.engine.drafters import LookupDrafter, MultiDrafter, SpecTree, TreeLookupDrafter, accept_tree


def test_lookup_proposes_what_followed_the_latest_match():
    ctx = [1, 2, 3, 4, 9, 9, 1, 2, 3, 5, 6, 7, 1, 2, 3]
    d = LookupDrafter(ctx, min_n=1, max_n=3)
    assert d.draft(3) == [5, 6, 7]            # the most recent earlier "1 2 3" was followed by 5 6 7
    d.commit([5, 6])
    assert d.draft(2) == [7, 1]               # suffix "3 5 6" -> "7 1"
    assert LookupDrafter([1, 2, 3]).draft(4) == []
    ref = LookupDrafter([7, 8], refs=[[0, 7, 8, 42, 43]])
    assert ref.draft(2) == [42, 43]           # retrieval from a reference corpus


class Fixed:
    def __init__(self, out):
        self.out, self.commits = out, []

    def draft(self, k):
        return self.out[:k]

    def commit(self, toks):
        self.commits.append(list(toks))


def test_multi_drafter_routes_to_the_better_member_and_probes():
    good, bad = Fixed([1, 2, 3]), Fixed([9, 9, 9])
    md = MultiDrafter([("bad", bad), ("good", good)], probe_every=4)
    picks = []
    for _ in range(12):
        d = md.draft(3)
        picks.append("good" if d == [1, 2, 3] else "bad")
        md.commit([1, 2, 3, 4])
    assert picks[:2] == ["bad", "good"]                       # every member tried once
    assert picks.count("good") >= 8 and "bad" in picks[2:]    # mostly good, probes the other
    st = {s["name"]: s for s in md.stats()}
    assert st["good"]["rate"] == 1.0 and st["bad"]["rate"] == 0.0
    assert good.commits[-1] == [1, 2, 3, 4] and bad.commits[-1] == [1, 2, 3, 4]


def test_tree_lookup_merges_continuations_into_a_trie():
    ctx = [5, 1, 2, 7, 8, 0, 1, 2, 7, 9, 0, 1, 2, 6, 6, 0, 1, 2]
    t = TreeLookupDrafter(ctx, width=3, min_n=2, max_n=2).propose(3)
    paths = sorted(tuple(t.tokens[i] for i in t.path(leaf)) for leaf in t.leaves())
    assert paths == [(6, 6, 0), (7, 8, 0), (7, 9, 0)]
    assert sum(1 for p in t.parent if p == -1) == 2           # "7" shared by two branches
    assert all(p < i for i, p in enumerate(t.parent))          # parents first


def test_accept_tree_commits_the_greedy_path():
    # root -> a(10) -> b(11) -> c(12);  root -> x(20)
    tree = SpecTree([10, 20, 11, 12], [-1, -1, 0, 2])
    # target greedy: after root 10, after a 11, after b 99 (rejects c), ...
    path, committed = accept_tree(tree, 10, [11, 0, 99, 5])
    assert path == [0, 2] and committed == [10, 11, 99]
    path, committed = accept_tree(tree, 20, [11, 3, 99, 5])
    assert path == [1] and committed == [20, 3]
    path, committed = accept_tree(tree, 7, [11, 3, 99, 5])
    assert path == [] and committed == [7]
    assert tree.depth(3) == 3
