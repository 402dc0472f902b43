"""Per-step breakdown of the decode loop: device time of one step against the GPU's idle gap between
steps (the host's share), for the synchronous loop and the device-resident one.

Runs the headline session (Qwen2.5-7B-arch Q4_K_M, 5 agents sharing an 8192-token prefix, +256 user
tokens and 128 greedy tokens per turn) through the engine, and brackets every decode graph replay
with CUDA events: ``device`` = end - start of a step, ``gap`` = start of step t - end of step t - 1
(time the GPU sat idle waiting for the host).  With N ranks (torchrun) every figure is the max over
ranks.

    python -m fak_b200.benchmarks.stepprof [--turns 2] [--warmup 3]
    torchrun --nproc-per-node N -m fak_b200.benchmarks.stepprof
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import time

import numpy as np
import torch


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen2.5-7b")
    ap.add_argument("--mix", default="q4_k_m")
    ap.add_argument("--agents", type=int, default=5)
    ap.add_argument("--prefix", type=int, default=8192)
    ap.add_argument("--user", type=int, default=256)
    ap.add_argument("--decode", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--turns", type=int, default=2, help="measured turns per loop mode")
    ap.add_argument("--modes", default="sync,async")
    ap.add_argument("--profile", type=int, default=0,
                    help="N > 0: also attribute N async decode steps to kernels (CUPTI activity through "
                         "torch.profiler; attribution only, the timings above are CUDA events)")
    args = ap.parse_args(argv)

    import torch.distributed as dist

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
    modes = args.modes.split(",")
    turns = args.warmup + args.turns * len(modes)
    max_ctx = (args.prefix + (turns + 1) * (args.user + args.decode) + 64 + 15) // 16 * 16
    ecfg = EngineConfig.from_env(max_batch=max(8, args.agents), cuda_graph=True,
                                 graph_batch_buckets=tuple(sorted({1, 2, 4, 8, args.agents})),
                                 max_prefill_tokens=max(args.prefix, args.agents * args.user), tp=world)
    eng = Engine.synthetic(cfg, args.mix, 0, ecfg, dev, max_context=max_ctx, tp_group=group)
    eng.warmup_graphs()
    rn = eng.runner
    marks: list[tuple[torch.cuda.Event, torch.cuda.Event]] = []

    def timed(fn):
        def wrap(*a, **k):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            out = fn(*a, **k)
            e1.record()
            marks.append((e0, e1))
            return out
        return wrap

    rn.replay_resident = timed(rn.replay_resident)
    rn.decode = timed(rn.decode)

    rng = np.random.default_rng(0)
    V = cfg.vocab_size
    prefix = rng.integers(0, V, args.prefix).tolist()
    hist = [list(prefix) for _ in range(args.agents)]
    eng.generate([prefix], max_new_tokens=1)

    def turn():
        reqs = []
        for a in range(args.agents):
            hist[a].extend(rng.integers(0, V, args.user).tolist())
            reqs.append(eng.add_request(hist[a], args.decode))
        eng.run_until_done(reqs)
        for a, r in enumerate(reqs):
            hist[a].extend(r.full_output)

    for _ in range(args.warmup):
        turn()
    results = {}
    for mode in modes:
        eng.ecfg.async_decode = mode == "async"
        dev_ms, gap_ms, wall = [], [], []
        for _ in range(args.turns):
            torch.cuda.synchronize()
            marks.clear()
            t0 = time.perf_counter()
            turn()
            torch.cuda.synchronize()
            wall.append(1000 * (time.perf_counter() - t0))
            steps = marks[-(args.decode - 1):]   # the turn's decode steps (the first token comes from prefill)
            dev_ms += [a.elapsed_time(b) for a, b in steps]
            gap_ms += [steps[i - 1][1].elapsed_time(steps[i][0]) for i in range(1, len(steps))]
        r = torch.tensor([statistics.median(dev_ms), statistics.median(gap_ms), statistics.mean(dev_ms),
                          statistics.mean(gap_ms), statistics.median(wall)], dtype=torch.float64, device=dev)
        if group is not None:
            dist.all_reduce(r, op=dist.ReduceOp.MAX)
        results[mode] = {"device_ms_per_step_median": round(float(r[0]), 4), "gap_ms_per_step_median": round(float(r[1]), 4),
                         "device_ms_per_step_mean": round(float(r[2]), 4), "gap_ms_per_step_mean": round(float(r[3]), 4),
                         "turn_wall_ms_median": round(float(r[4]), 2)}
    if args.profile > 0:
        results["kernels_us_per_step"] = _kernel_profile(eng, turn, args, group, world)
    if rank == 0:
        print(json.dumps({"bench": "stepprof", "model": f"{cfg.name}-arch {args.mix}", "n_gpus": world,
                          "agents": args.agents, "prefix": args.prefix, "decode_steps_per_turn": args.decode - 1,
                          "turns_per_mode": args.turns, "max_over_ranks": True, **results}), flush=True)
    eng.shutdown()
    if group is not None:
        pdist.shutdown()


def _kernel_profile(eng, turn, args, group, world) -> dict:
    """Per-kernel device time of decode steps (us per step, max over ranks), from a profiled turn."""
    import torch.distributed as dist
    from torch.profiler import ProfilerActivity, profile
    eng.ecfg.async_decode = True
    rn = eng.runner
    n_steps = [0]
    real = rn.replay_resident

    def counted(*a, **k):
        n_steps[0] += 1
        return real(*a, **k)
    rn.replay_resident = counted
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        turn()
        torch.cuda.synchronize()
    rn.replay_resident = real
    agg: dict[str, float] = {}
    seq: list[tuple[float, str, float]] = []
    for ev in prof.events():
        if ev.device_type.name != "CUDA":
            continue
        name = ev.name.replace("void ", "").replace("(anonymous namespace)::", "").replace("<unnamed>::", "")
        name = name.split("(")[0][:48] or ev.name[:48]
        agg[name] = agg.get(name, 0.0) + ev.device_time
        seq.append((ev.time_range.start, name, ev.device_time))
    # one decode step in launch order (a step starts with the embedding gather): the third one
    seq.sort()
    starts = [i for i, (_, n, _) in enumerate(seq) if n.startswith("k_embed")]
    step_trace = []
    if len(starts) >= 4:
        a, b = starts[2], starts[3]
        step_trace = [(n, round(t, 2)) for _, n, t in seq[a:b]]
    # decode steps only: subtract nothing, report per decode step of the profiled turn
    steps = max(1, n_steps[0])
    per = {k: v / steps for k, v in agg.items()}
    if group is not None:
        allp = [None] * world
        dist.all_gather_object(allp, per, group=group)
        keys = set().union(*[set(p) for p in allp])
        per = {k: max(p.get(k, 0.0) for p in allp) for k in keys}
    top = sorted(per.items(), key=lambda kv: -kv[1])[:16]
    out = {k: round(v, 2) for k, v in top}
    if step_trace:   # this rank's (rank 0's) kernels of one step: the first layer, and the step's tail
        out["_step_trace_first_layer_and_tail"] = step_trace[:16] + [("...", 0.0)] + step_trace[-8:]
        out["_step_kernels"] = len(step_trace)
        out["_step_us_sum"] = round(sum(t for _, t in step_trace), 1)
    return out


if __name__ == "__main__":
    main()
