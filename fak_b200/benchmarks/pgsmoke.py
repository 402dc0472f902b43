"""Multi-process collective smoke test, one rank per GPU (reference: cmd/pgsmoke -- NCCL process
group init and an all-reduce whose result every rank checks).

Each rank fills a buffer with values that make the exact sum known (rank r contributes r + 1 in
every element, scaled by a position pattern), then runs

1. an NCCL all-reduce through ``torch.distributed`` (the baseline path), and
2. the in-kernel peer-memory all-reduce (``k_p2p_allreduce_add`` over CUDA IPC peer buffers, the
   collective the decode path fuses into its GEMV epilogues),

and checks both against the exact sum on every rank (integers small enough to be exact in fp32).
Timings are CUDA events, max over ranks.  Rank 0 prints one JSON line.

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 -m fak_b200.benchmarks.pgsmoke
"""
from __future__ import annotations

import argparse
import json
import os

import torch


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--elems", type=int, default=1 << 20)
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args(argv)
    import torch.distributed as dist

    from fak_b200.ops._ext import ext
    from fak_b200.parallel import dist as pdist
    from fak_b200.parallel.p2p import AR_CTAS, PeerBuffer
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = pdist.init(world, rank, local)
    n = args.elems // 4 * 4
    pattern = (torch.arange(n, device=dev, dtype=torch.int64) % 97).float()
    mine = pattern * (rank + 1)
    want = pattern * (world * (world + 1) // 2)

    def timed(fn) -> float:
        fn()
        torch.cuda.synchronize()
        dist.barrier(group=group)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.iters):
            fn()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / args.iters], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        return float(t)

    # 1. NCCL
    buf = mine.clone()
    dist.all_reduce(buf, group=group)
    nccl_ok = bool(torch.equal(buf, want))
    nccl_ms = timed(lambda: dist.all_reduce(buf, group=group))
    # 2. in-kernel peer all-reduce: x (zero) += sum of every rank's partial in its peer buffer
    flags_bytes = 4 * 64 * 8
    pb = PeerBuffer(flags_bytes + 4 * n, group, dev)
    peers = torch.tensor(pb.ptrs, dtype=torch.int64)
    part = pb.buf[flags_bytes:flags_bytes + 4 * n].view(torch.float32)
    part.copy_(mine)
    counters = torch.zeros(64, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    x = torch.zeros(n, device=dev)
    torch.cuda.synchronize()
    dist.barrier(group=group)
    ext().p2p_allreduce_add(peers, flags_bytes, x, n, 0, 0, rank, counters, err, AR_CTAS, 0)
    torch.cuda.synchronize()
    p2p_ok = bool(torch.equal(x, want)) and int(err.item()) == 0
    p2p_ms = timed(lambda: ext().p2p_allreduce_add(peers, flags_bytes, x, n, 0, 0, rank, counters, err, AR_CTAS, 0))
    err_word = int(err.item())
    oks = torch.tensor([int(nccl_ok), int(p2p_ok)], device=dev)
    dist.all_reduce(oks, op=dist.ReduceOp.MIN, group=group)
    pb.close()
    if rank == 0:
        nbytes = 4 * n
        print(json.dumps({"bench": "pgsmoke", "world": world, "elems": n, "nccl_ok": bool(oks[0]),
                          "p2p_ok": bool(oks[1]), "p2p_error_word": err_word, "nccl_ms": round(nccl_ms, 4),
                          "p2p_ms": round(p2p_ms, 4),
                          "nccl_busbw_gbs": round(2 * (world - 1) / world * nbytes / nccl_ms / 1e6, 1),
                          "max_over_ranks": True}), flush=True)
    pdist.shutdown()
    return 0 if bool(oks.min()) else 1


if __name__ == "__main__":
    raise SystemExit(main())
