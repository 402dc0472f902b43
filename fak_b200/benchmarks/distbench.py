"""Decode / prefill throughput of one model over N ranks (tensor / expert parallel), timed on the device
with CUDA events and reported as the max over ranks.

Covers the benchmark configurations that are not the multi-agent headline:

* ``--model qwen3-30b-a3b --mix q8_0 --batch 64 --prefill 4096 --prefill-seqs 8``: the MoE config, its
  128 experts split into expert bands over the ranks (expert parallel), batch-64 decode and an
  8 x 4096-token prefill;
* ``--model qwen2.5-32b --spec-k 4 --batch 1``: self-speculative decode (draft = the first 4 layers +
  LM head), reporting accepted tokens per second and the verify-step latency;
* any dense model at TP = N with ``--batch`` lanes over ``--ctx`` tokens of context.

    torchrun --nproc-per-node N -m fak_b200.benchmarks.distbench --model qwen3-30b-a3b --mix q8_0 \\
        --batch 64 --ctx 256 --prefill 4096 --prefill-seqs 8
"""
from __future__ import annotations

import argparse
import json
import os
import time

import numpy as np
import torch


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3-30b-a3b")
    ap.add_argument("--mix", default="q8_0")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--ctx", type=int, default=256, help="prompt tokens per decode lane")
    ap.add_argument("--steps", type=int, default=32, help="timed decode steps")
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--prefill", type=int, default=0, help="tokens per prefill sequence (0: no prefill timing)")
    ap.add_argument("--prefill-seqs", type=int, default=1)
    ap.add_argument("--spec-k", type=int, default=0)
    ap.add_argument("--draft-layers", type=int, default=4)
    ap.add_argument("--drafter", default="self")
    args = ap.parse_args(argv)

    import torch.distributed as dist

    from fak_b200.config import EngineConfig, preset
    from fak_b200.engine import Engine
    from fak_b200.models.runner import PrefillMeta
    from fak_b200.parallel import dist as pdist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = pdist.init(world, rank, local) if world > 1 else None
    cfg = preset(args.model)
    B = args.batch
    new = args.steps + args.warmup + 2
    max_ctx = (max(args.ctx + new * (args.spec_k + 1) + 64, args.prefill + 16) + 15) // 16 * 16
    buckets = tuple(b for b in (1, 2, 4, 8, 16, 32, 64) if b <= max(B * (args.spec_k + 1), 8)) or (B,)
    ecfg = EngineConfig.from_env(max_batch=max(B * (args.spec_k + 1), 8), cuda_graph=True, graph_batch_buckets=buckets,
                                 max_prefill_tokens=max(4096, args.prefill * args.prefill_seqs, B * args.ctx),
                                 spec_k=args.spec_k, spec_draft_layers=args.draft_layers, spec_drafter=args.drafter,
                                 tp=world)
    t0 = time.perf_counter()
    eng = Engine.synthetic(cfg, args.mix, 0, ecfg, dev, max_context=max_ctx, tp_group=group)
    eng.warmup_graphs()
    load_s = time.perf_counter() - t0

    def max_ranks(vals):
        t = torch.tensor(vals, dtype=torch.float64, device=dev)
        if group is not None:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.tolist()

    rng = np.random.default_rng(0)
    reqs = [eng.add_request(rng.integers(0, cfg.vocab_size, args.ctx).tolist(), new) for _ in range(B)]
    while eng.prefilling or eng.waiting:
        eng._admit()
        eng._run_prefill()
    for _ in range(args.warmup):
        eng._run_decode()
    eng._drain()
    torch.cuda.synchronize()
    s0 = dict(eng.stats)
    if group is not None:
        dist.barrier(group=group)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        eng._run_decode()
    e1.record()
    eng._drain()
    torch.cuda.synchronize()
    dec_ms, = max_ranks([e0.elapsed_time(e1)])
    toks = eng.stats["decode_tokens"] - s0["decode_tokens"]
    out = {"bench": "distbench", "model": f"{cfg.name}-arch {args.mix}", "n_gpus": world,
           "parallelism": ("ep" if cfg.is_moe else "tp") + str(world), "batch": B, "ctx": args.ctx,
           "decode_steps": args.steps, "decode_ms_per_step": round(dec_ms / args.steps, 4),
           "max_over_ranks": True, "load_s": round(load_s, 1)}
    if args.spec_k:
        emitted = sum(len(r.full_output) for r in reqs)
        steps = eng.stats.get("spec_steps", 0) - s0.get("spec_steps", 0)
        acc = eng.stats.get("spec_accepted", 0) - s0.get("spec_accepted", 0)
        prop = eng.stats.get("spec_proposed", 0) - s0.get("spec_proposed", 0)
        out.update({"spec_k": args.spec_k, "drafter": args.drafter, "verify_steps": steps,
                    "verify_step_ms": round(dec_ms / max(1, steps), 4), "acceptance": round(acc / max(1, prop), 4),
                    "accepted_tok_s": round((acc + steps * B) * 1000.0 / dec_ms, 1), "emitted_total": emitted})
    else:
        out["decode_tok_s"] = round(toks * 1000.0 / dec_ms, 1)
    for r in reqs:
        r.finished = True
    eng.running.clear()
    if args.prefill:
        L, S = args.prefill, args.prefill_seqs
        T = L * S
        ids = torch.from_numpy(rng.integers(0, cfg.vocab_size, T).astype(np.int32)).to(dev)
        npg = (L + 15) // 16
        pages = [eng.pool.alloc(npg) for _ in range(S)]
        pos = torch.arange(L, dtype=torch.int32, device=dev).repeat(S)
        pg = torch.tensor(pages, dtype=torch.int64, device=dev)
        seq = torch.arange(S, device=dev).repeat_interleave(L)
        slot = (pg[seq, pos.long() // 16] * 16 + pos.long() % 16).int()
        meta = PrefillMeta.build([L] * S, [0] * S, dev)
        last = (torch.arange(S, dtype=torch.int32, device=dev) + 1) * L - 1
        eng.runner.prefill(ids, pos, slot, pg.int(), meta, last)
        torch.cuda.synchronize()
        if group is not None:
            dist.barrier(group=group)
        e0.record()
        n = 2
        for _ in range(n):
            eng.runner.prefill(ids, pos, slot, pg.int(), meta, last)
        e1.record()
        torch.cuda.synchronize()
        pms, = max_ranks([e0.elapsed_time(e1) / n])
        out.update({"prefill_seqs": S, "prefill_tokens": T, "prefill_ms": round(pms, 3),
                    "prefill_tok_s": round(T * 1000.0 / pms, 1)})
        for p_ in pages:
            eng.pool.release(p_)
    if rank == 0:
        print(json.dumps(out), flush=True)
    eng.shutdown()
    if group is not None:
        pdist.shutdown()


if __name__ == "__main__":
    main()
