"""Self-speculative decoding benchmark (the Qwen2.5-32B spec-decode configuration).

The draft is the target's first ``--draft-layers`` layers plus its LM head, sharing the target's KV
pages; each verify step checks ``--k`` drafted tokens per sequence in one target forward.  Reports
accepted (emitted) tok/s, the verify-step latency and the acceptance rate, against plain greedy
decoding of the same prompts on the same engine (reference: spec.SpeculativeGreedy,
internal/spec/spec.go:214-300; BENCHMARK-AUTHORITY.md:36 reports tokens per verify).

    python -m fak_b200.benchmarks.specbench --model qwen2.5-32b --batch 1 --prompt 4096 --decode 1024
"""
from __future__ import annotations

import argparse
import json

import numpy as np
import torch


def _decode_all(eng, reqs) -> float:
    """Prefill everything, then time the decode phase to completion with CUDA events (ms)."""
    while eng.prefilling or eng.waiting:
        eng._admit()
        eng._run_prefill()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    while eng.running:
        eng._run_decode()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen2.5-32b")
    ap.add_argument("--mix", default="q4_k_m")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--prompt", type=int, default=4096)
    ap.add_argument("--decode", type=int, default=1024)
    ap.add_argument("--k", type=int, default=4)
    ap.add_argument("--draft-layers", type=int, default=4)
    ap.add_argument("--seed", type=int, default=0)
    args = ap.parse_args(argv)

    from fak_b200.config import EngineConfig, preset
    from fak_b200.engine import Engine

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = preset(args.model)
    B = args.batch
    V = B * (args.k + 1)  # verify lanes
    buckets = tuple(sorted({1, 2, 4, 8, B, V} | ({16} if V > 8 else set())))
    max_ctx = (args.prompt + args.decode + args.k + 64 + 15) // 16 * 16
    ecfg = EngineConfig(max_batch=max(V, 8), cuda_graph=True, graph_batch_buckets=buckets,
                        max_prefill_tokens=max(4096, args.prompt), spec_k=args.k,
                        spec_draft_layers=args.draft_layers, radix_cache=False)
    eng = Engine.synthetic(cfg, args.mix, args.seed, ecfg, dev, max_context=max_ctx)
    eng.warmup_graphs()
    rng = np.random.default_rng(args.seed)
    prompts = [rng.integers(0, cfg.vocab_size, args.prompt).tolist() for _ in range(B)]

    # plain greedy decode (same engine, speculation off)
    eng.ecfg.spec_k = 0
    base = [eng.add_request(p, args.decode) for p in prompts]
    base_ms = _decode_all(eng, base)
    base_tokens = sum(len(r.output) for r in base)

    eng.ecfg.spec_k = args.k
    s0 = dict(eng.stats)
    spec = [eng.add_request(p, args.decode) for p in prompts]
    spec_ms = _decode_all(eng, spec)
    spec_tokens = sum(len(r.output) for r in spec)
    steps = eng.stats.get("spec_steps", 0) - s0.get("spec_steps", 0)
    proposed = eng.stats.get("spec_proposed", 0) - s0.get("spec_proposed", 0)
    accepted = eng.stats.get("spec_accepted", 0) - s0.get("spec_accepted", 0)
    same = all(a.output == b.output for a, b in zip(base, spec))
    print(json.dumps({
        "model": args.model, "batch": B, "prompt": args.prompt, "decode": args.decode, "k": args.k,
        "draft_layers": args.draft_layers,
        "accepted_tok_s": round(spec_tokens * 1000 / spec_ms, 1),
        "greedy_tok_s": round(base_tokens * 1000 / base_ms, 1),
        "speedup": round(base_ms / spec_ms * spec_tokens / max(1, base_tokens), 3),
        "verify_steps": steps, "verify_step_ms": round(spec_ms / max(1, steps), 3),
        "tokens_per_verify": round(spec_tokens / max(1, steps) / B, 3),
        "acceptance": round(accepted / max(1, proposed), 4),
        "matches_greedy": same,
        "weights": "random-init N(0,0.02), synthetic " + args.mix,
    }), flush=True)


if __name__ == "__main__":
    main()
