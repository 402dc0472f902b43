"""Tensor-parallel agreement check (reference: cmd/tpcheck).

Every rank builds the same synthetic model sharded TP=world and greedily decodes the same
prompts; rank 0 also runs an unsharded (TP=1) engine on its GPU and compares the tokens.

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \\
        -m fak_b200.benchmarks.tpcheck --model tiny-qwen2
"""
from __future__ import annotations

import argparse
import json
import os

import numpy as np
import torch


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="tiny-qwen2")
    ap.add_argument("--mix", default="q4_k_m", help="q4_k_m, q8_0 (MoE checkpoints use q8_0)")
    ap.add_argument("--new", type=int, default=12)
    ap.add_argument("--graphs", type=int, default=1)
    ap.add_argument("--fused", type=int, default=1, help="1: in-kernel P2P collectives, 0: NCCL")
    args = ap.parse_args(argv)
    from fak_b200.config import EngineConfig, preset
    from fak_b200.engine import Engine
    from fak_b200.parallel import dist as pdist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = pdist.init(world, rank, local) if world > 1 else None
    cfg = preset(args.model)
    ecfg = EngineConfig(max_batch=8, kv_pages=1024, cuda_graph=bool(args.graphs), graph_batch_buckets=(1, 2, 4),
                        fused_collectives=bool(args.fused))
    rng = np.random.default_rng(7)
    prompts = [rng.integers(0, cfg.vocab_size, n).tolist() for n in (37, 90, 5)]
    eng = Engine.synthetic(cfg, args.mix, 3, ecfg, dev, max_context=2048, tp_group=group, std=0.05)
    eng.warmup_graphs()
    outs = eng.generate(prompts, args.new)
    coll_err = eng.runner.coll.check() if hasattr(eng.runner.coll, "check") else 0
    eng.shutdown()
    result = {"rank": rank, "world": world, "tp_outputs": outs, "collective_error": coll_err}
    if rank == 0:
        ref = Engine.synthetic(cfg, args.mix, 3, EngineConfig(max_batch=8, kv_pages=1024, cuda_graph=False), dev,
                               max_context=2048, std=0.05)
        want = ref.generate(prompts, args.new)
        prefix_agree = []
        for o, w in zip(outs, want):
            k = 0
            while k < len(o) and o[k] == w[k]:
                k += 1
            prefix_agree.append(k)
        result.update({"tp1_outputs": want, "prefix_agree": prefix_agree,
                       "ok": all(k >= min(4, args.new) for k in prefix_agree) and coll_err == 0})
        print(json.dumps(result), flush=True)
    if group is not None:
        pdist.shutdown()


if __name__ == "__main__":
    main()
