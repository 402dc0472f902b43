"""Session checkpoint / restore of a serving engine.

A checkpoint records what the engine would need to continue serving the same agents:

* the radix prefix cache as token sequences (every root-to-leaf path), optionally with the bf16
  K/V of their pages (``include_kv``) so a restore needs no recompute;
* the requests in flight: tokens so far, generated output, remaining budget, sampling settings.

Restoring into an engine of the same model re-inserts the cached sequences (copying saved K/V into
freshly allocated pages, or re-prefilling them when only tokens were saved) and queues the
requests again; their KV is recomputed from the radix cache on admission (cheap: their prefixes
are cached).  The file is a ``torch.save`` dictionary.

Reference: portable session images (internal/sessionimage, tar ``.faksession``), KV clone and
paged swap (internal/model/kvcache.go:181, paged_swap.go) and ``--session-state`` (serve.go:162).
"""
from __future__ import annotations

import dataclasses

import torch

from .sampling import SamplingParams

FORMAT = "fak-b200-session/v1"


def save_session(engine, path: str, include_kv: bool = False) -> dict:
    seqs = engine.radix.sequences() if engine.radix is not None else []
    kv = None
    if include_kv and seqs:
        kv = []
        for toks, pages in seqs:
            idx = torch.tensor(pages, dtype=torch.long, device=engine.kv.k.device)
            kv.append((engine.kv.k[:, idx].cpu(), engine.kv.v[:, idx].cpu()))
    reqs = []
    for r in list(engine.running) + list(engine.prefilling) + list(engine.swapped) + list(engine.waiting):
        if r.finished:
            continue
        reqs.append({"tokens": list(r.tokens), "output": list(r.full_output),
                     "remaining": r.max_new_tokens - len(r.output),
                     "sampling": dataclasses.asdict(dataclasses.replace(r.sampling, mask=None)),
                     "stop_ids": sorted(r.stop_ids)})
    state = {"format": FORMAT, "model": engine.cfg.name, "n_layers": engine.cfg.n_layers,
             "page_size": engine.ecfg.page_size, "cache": [t for t, _ in seqs], "kv": kv, "requests": reqs}
    torch.save(state, path)
    return {"cached_sequences": len(seqs), "requests": len(reqs), "kv": include_kv}


def load_session(engine, path: str) -> list:
    """Restore a checkpoint; returns the re-queued requests (in checkpoint order)."""
    state = torch.load(path, map_location="cpu", weights_only=False)
    if state.get("format") != FORMAT:
        raise ValueError(f"{path}: not a {FORMAT} checkpoint")
    if state["n_layers"] != engine.cfg.n_layers or state["page_size"] != engine.ecfg.page_size:
        raise ValueError("checkpoint was taken on a different model or page size")
    ps = engine.ecfg.page_size
    if engine.radix is not None:
        if state["kv"] is not None:
            for toks, (k, v) in zip(state["cache"], state["kv"]):
                pages = engine._alloc(len(toks) // ps)
                idx = torch.tensor(pages, dtype=torch.long, device=engine.kv.k.device)
                engine.kv.k[:, idx] = k.to(engine.kv.k.device)
                engine.kv.v[:, idx] = v.to(engine.kv.v.device)
                engine.radix.insert(toks, pages)
                engine.pool.release(pages)
        else:
            for toks in state["cache"]:  # recompute: prefill the sequence (one throwaway token)
                if len(toks) + 1 <= engine.max_context:
                    engine.generate([toks], max_new_tokens=1)
    out = []
    for q in state["requests"]:
        sp = SamplingParams(**q["sampling"])
        r = engine.add_request(q["tokens"], max(1, q["remaining"]), sp, q["stop_ids"])
        r.output_before_preempt = list(q["output"])
        out.append(r)
    return out
