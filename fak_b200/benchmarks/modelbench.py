"""Decode / prefill microbenchmark of the model runner (reference: cmd/modelbench).

Builds a random-init model of a named architecture on the GPU, prefills ``--batch``
sequences of ``--ctx`` tokens, then times ``--steps`` decode steps (CUDA graph by default)
with CUDA events, and one prefill chunk.  Used for kernel profiling:

    python -m fak_b200.benchmarks.modelbench --model qwen2.5-7b --batch 5 --ctx 9000 --steps 20
"""
from __future__ import annotations

import argparse
import json
import time

import numpy as np
import torch


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen2.5-7b")
    ap.add_argument("--mix", default="q4_k_m")
    ap.add_argument("--batch", type=int, default=5)
    ap.add_argument("--ctx", type=int, default=9000)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--prefill", type=int, default=1280, help="tokens per sequence in the timed prefill chunk")
    ap.add_argument("--prefill-seqs", type=int, default=1, help="sequences in the timed prefill chunk")
    ap.add_argument("--eager", action="store_true", help="no CUDA graph (one launch per op)")
    ap.add_argument("--decode-only", action="store_true")
    args = ap.parse_args(argv)

    from fak_b200.config import EngineConfig, preset
    from fak_b200.engine import Engine
    from fak_b200.models.runner import PrefillMeta
    from fak_b200.ops import kernels as K

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = preset(args.model)
    B = args.batch
    # the RoPE tables and block tables cover both the decode contexts and the timed prefill
    max_ctx = (max(args.ctx + args.steps + args.warmup + 64, args.prefill) + 15) // 16 * 16
    ecfg = EngineConfig.from_env(max_batch=max(B, 8), cuda_graph=not args.eager, graph_batch_buckets=(B,),
                        max_prefill_tokens=max(4096, args.prefill * args.prefill_seqs))
    eng = Engine.synthetic(cfg, args.mix, 0, ecfg, dev, max_context=max_ctx)
    if not args.eager:
        eng.warmup_graphs()
    rng = np.random.default_rng(0)
    # B independent contexts (no sharing), prefilled through the engine
    reqs = [eng.add_request(rng.integers(0, cfg.vocab_size, args.ctx).tolist(), args.steps + args.warmup + 2)
            for _ in range(B)]
    while eng.prefilling or eng.waiting:
        eng._admit()
        eng._run_prefill()
    torch.cuda.synchronize()
    for _ in range(args.warmup):
        eng._run_decode()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    l0 = K.launches()
    e0.record()
    t0 = time.perf_counter()
    torch.cuda.nvtx.range_push("fak_decode")
    for _ in range(args.steps):
        eng._run_decode()
    torch.cuda.nvtx.range_pop()
    e1.record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    dms = e0.elapsed_time(e1) / args.steps
    out = {"model": args.model, "batch": B, "ctx": args.ctx, "decode_ms_per_step": round(dms, 4),
           "decode_tok_s": round(B * 1000 / dms, 1), "wall_ms_per_step": round(1000 * wall / args.steps, 4),
           "launches_per_step": (K.launches() - l0) / args.steps,
           "weight_bytes": eng.weights.nbytes()}
    if not args.decode_only:
        # --prefill-seqs independent sequences of --prefill tokens in one chunk
        L, S = args.prefill, args.prefill_seqs
        T = L * S
        ids = torch.from_numpy(rng.integers(0, cfg.vocab_size, T).astype(np.int32)).to(dev)
        npg = (L + 15) // 16
        pages = [eng.pool.alloc(npg) for _ in range(S)]
        pos = torch.arange(L, dtype=torch.int32, device=dev).repeat(S)
        pg = torch.tensor(pages, dtype=torch.int64, device=dev)                 # [S, npg]
        seq = torch.arange(S, device=dev).repeat_interleave(L)
        slot = (pg[seq, pos.long() // 16] * 16 + pos.long() % 16).int()
        bt = pg.int()
        meta = PrefillMeta.build([L] * S, [0] * S, dev)
        last = (torch.arange(S, dtype=torch.int32, device=dev) + 1) * L - 1
        for _ in range(2):
            eng.runner.prefill(ids, pos, slot, bt, meta, last)
        torch.cuda.synchronize()
        e0.record()
        n = 3
        torch.cuda.nvtx.range_push("fak_prefill")
        for _ in range(n):
            eng.runner.prefill(ids, pos, slot, bt, meta, last)
        torch.cuda.nvtx.range_pop()
        e1.record()
        torch.cuda.synchronize()
        pms = e0.elapsed_time(e1) / n
        flops = 2.0 * T * (cfg.param_count() - cfg.vocab_size * cfg.d_model)
        out.update({"prefill_seqs": S, "prefill_tokens": T, "prefill_ms": round(pms, 3), "prefill_tok_s": round(T * 1000 / pms, 1),
                    "prefill_linear_tflops": round(flops / pms / 1e9, 1)})
    print(json.dumps(out), flush=True)
    return out


if __name__ == "__main__":
    main()
