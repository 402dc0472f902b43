"""Cost of the all-reduce fused into the decode GEMV epilogue, in isolation: one row-parallel
projection (rows = d_model, this rank's K slice) at decode batch B, launched back to back inside a
CUDA graph, CUDA events, max over ranks.  Variants:

* ``plain``  -- the GEMV with a residual add and no all-reduce (the compute floor);
* ``fused``  -- the GEMV whose epilogue pushes each tile to every rank and sums (``tgemv`` ``ar``);
* ``p2p``    -- the GEMV into a partial buffer, then the one-shot peer-memory all-reduce kernel;
* ``nccl``   -- the GEMV into a partial buffer, then an NCCL all-reduce and an add (eager launches).

Several weight copies rotate so every launch streams its weights from DRAM.

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 -m fak_b200.benchmarks.arbench \\
        --rows 3584 --cols 1792 --batch 5
"""
from __future__ import annotations

import argparse
import json
import os

import torch


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=3584)
    ap.add_argument("--cols", type=int, default=0, help="this rank's K slice (default 3584 / world)")
    ap.add_argument("--qtype", type=int, default=12)
    ap.add_argument("--batch", type=int, default=5)
    ap.add_argument("--iters", type=int, default=100)
    ap.add_argument("--variants", default="plain,fused,p2p,nccl")
    args = ap.parse_args(argv)
    import torch.distributed as dist

    from fak_b200.models.weights import QuantWeight
    from fak_b200.ops import kernels as K
    from fak_b200.ops import quant as dq
    from fak_b200.ops._ext import ext
    from fak_b200.parallel import dist as pdist
    from fak_b200.parallel.p2p import AR_CTAS, MAX_CTAS, MAX_W, PeerBuffer, _align, ar_slot_bytes

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = pdist.init(world, rank, local)
    N, B = args.rows, args.batch
    Kc = args.cols or 3584 // world
    n_copies = max(2, int(400e6 // (N * dq.row_bytes(args.qtype, Kc))) + 1)
    ws = []
    for i in range(n_copies):
        raw = dq.synth_quantized((N, Kc), args.qtype, 77 + 13 * rank + i, 0.02, device="cuda")
        ws.append(QuantWeight.from_rows(raw.view(N, -1), args.qtype, Kc, dev).pack())
        ws[-1].buf = None
    act = K.ActQ(max(8, B), Kc, dev)
    K.quant_act(torch.randn(B, Kc, device=dev), act)
    K.tgemv_workspace(dev, ws)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    K.register_error_word(dev, err)

    # peer buffer: barrier flags and partials of the unfused path, line slots of the fused path
    T = (N + 15) // 16
    off = 0
    flags_off = off
    off = _align(off + MAX_CTAS * MAX_W * 4)
    parts_off = off
    off = _align(off + B * N * 4)
    arparts_off = off
    off = _align(off + ar_slot_bytes(T))
    mem = PeerBuffer(off, group, dev)
    peers = torch.tensor(mem.ptrs, dtype=torch.int64)
    epochs = torch.zeros(T, dtype=torch.int32, device=dev)
    counters = torch.zeros(MAX_CTAS, dtype=torch.int32, device=dev)
    x = torch.zeros(B, N, device=dev)
    part = mem.buf[parts_off:parts_off + B * N * 4].view(torch.float32).view(B, N)
    ar = (peers, rank, arparts_off, epochs, 0)

    def one(v: str, w) -> None:
        if v == "plain":
            K.gemv(w, act, B, x, None, K.EPI_ADD)
        elif v == "fused":
            K.gemv(w, act, B, x, None, K.EPI_ADD, ar=ar)
        elif v == "p2p":
            K.gemv(w, act, B, part, None, K.EPI_STORE)
            ext().p2p_allreduce_add(peers, parts_off, x, B * N, flags_off, 0, rank, counters, err, AR_CTAS, 0)
        else:
            K.gemv(w, act, B, part, None, K.EPI_STORE)
            dist.all_reduce(part, group=group)
            x.add_(part)

    out = {"bench": "arbench", "n_gpus": world, "rows": N, "cols_per_rank": Kc, "batch": B, "qtype": args.qtype,
           "weight_mb_per_rank": round(ws[0].tp.numel() / 1e6, 2), "us_per_launch_max_over_ranks": {},
           "us_per_launch_by_rank": {}}
    for v in args.variants.split(","):
        for i in range(3):
            one(v, ws[i % n_copies])
        torch.cuda.synchronize()
        dist.barrier(group=group)
        g = None
        if v != "nccl":   # the graphs hold no NCCL call
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for i in range(args.iters):
                    one(v, ws[i % n_copies])
            g.replay()
            torch.cuda.synchronize()
            dist.barrier(group=group)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        if g is not None:
            g.replay()
        else:
            for i in range(args.iters):
                one(v, ws[i % n_copies])
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) * 1e3 / args.iters], dtype=torch.float64, device=dev)
        allt = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(allt, t, group=group)
        out["us_per_launch_max_over_ranks"][v] = round(max(float(a) for a in allt), 2)
        out["us_per_launch_by_rank"][v] = [round(float(a), 2) for a in allt]
        del g
        dist.barrier(group=group)
    out["error_word"] = int(err.item())
    if rank == 0:
        print(json.dumps(out), flush=True)
    mem.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
