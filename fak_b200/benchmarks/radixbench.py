"""Radix prefix-cache hit rate on synthetic shared-prefix workloads (hardware independent, CPU).

Each workload is a list of requests (token-id prompts whose shared prefixes are literally the same
ids); requests run in order through the engine's radix cache (lookup, allocate the missed pages,
insert, release -- exactly what the engine does per request).  Reports the cache hit rate (prompt
tokens served from cache) and the prefill-token speedup against a cold, cache-less baseline.

Workloads (the shapes of the reference's radixbench, cmd/radixbench/main.go:98-181):
  few_shot  N questions after one P-token preamble;
  chat      multi-turn conversations whose every turn re-sends the history;
  tree      tree-of-thought: every root-to-leaf path of a branching tree of S-token thoughts;
  agents    C agents sharing a P-token system prefix, each taking T steps that append a segment.

    python -m fak_b200.benchmarks.radixbench [--page-size 16] [--native 1]
"""
from __future__ import annotations

import argparse
import itertools
import json

import numpy as np


def few_shot(rng, n=64, preamble=2048, q=64):
    pre = rng.integers(0, 32000, preamble).tolist()
    return [pre + rng.integers(0, 32000, q).tolist() for _ in range(n)]


def chat(rng, convs=8, turns=8, user=96, reply=160):
    reqs = []
    hist = [rng.integers(0, 32000, 256).tolist() for _ in range(convs)]
    for _ in range(turns):
        for c in range(convs):
            hist[c] = hist[c] + rng.integers(0, 32000, user).tolist()
            reqs.append(list(hist[c]))
            hist[c] = hist[c] + rng.integers(0, 32000, reply).tolist()
    return reqs


def tree(rng, fanout=3, depth=4, step=128, root=512):
    base = rng.integers(0, 32000, root).tolist()
    reqs = []

    def walk(prefix, d):
        if d == depth:
            reqs.append(prefix)
            return
        for _ in range(fanout):
            walk(prefix + rng.integers(0, 32000, step).tolist(), d + 1)
    walk(base, 0)
    return reqs


def agents(rng, c=5, steps=50, prefix=8192, seg=384):
    sysp = rng.integers(0, 32000, prefix).tolist()
    hist = [list(sysp) for _ in range(c)]
    reqs = []
    for _ in range(steps):
        for a in range(c):
            hist[a] = hist[a] + rng.integers(0, 32000, seg).tolist()
            reqs.append(list(hist[a]))
    return reqs


WORKLOADS = {"few_shot": few_shot, "chat": chat, "tree": tree, "agents": agents}


def run(reqs, page_size: int, native: bool) -> dict:
    from fak_b200.kv import radix as R
    if native:
        import torch  # noqa: F401
        from fak_b200 import _cpu
        Pool, Cache = _cpu.PagePool, _cpu.RadixCache
    else:
        Pool, Cache = R.PyPagePool, R.PyRadixCache
    total_pages = sum(-(-len(r) // page_size) for r in reqs) + 16
    pool = Pool(total_pages, 1)
    rc = Cache(pool, page_size)
    prompt, hit = 0, 0
    for r in reqs:
        n, pages = rc.lookup(r, len(r) - 1)  # the last token is always computed (its logits)
        new = pool.alloc(-(-len(r) // page_size) - len(pages))
        rc.insert(r, pages + new)
        pool.release(pages + new)
        prompt += len(r)
        hit += n
    return {"requests": len(reqs), "prompt_tokens": prompt, "hit_tokens": hit,
            "hit_rate": round(hit / prompt, 4), "prefill_speedup": round(prompt / max(1, prompt - hit), 2)}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--page-size", type=int, default=16)
    ap.add_argument("--native", type=int, default=1)
    ap.add_argument("--seed", type=int, default=0)
    args = ap.parse_args(argv)
    native = bool(args.native)
    if native:
        try:
            import torch  # noqa: F401  (the extension links against its libraries)
            from fak_b200 import _cpu  # noqa: F401
        except ImportError:
            native = False
    for name, fn in WORKLOADS.items():
        reqs = fn(np.random.default_rng(args.seed))
        print(json.dumps({"workload": name, "page_size": args.page_size, "impl": "native" if native else "python",
                          **run(reqs, args.page_size, native)}), flush=True)


if __name__ == "__main__":
    main()
