"""Cost of the prefill all-reduce of a row-parallel projection, in isolation: x[M, N] += all-reduce
over ranks of a[M, K] . w[N, K]^T (this rank's K slice), CUDA events around ``--iters`` eager
iterations, max over ranks.  Variants:

* ``gemm``      -- the tcgen05 GEMM alone into a local fp32 buffer (the compute floor);
* ``fused``     -- the GEMM whose epilogue stores each tile into its owner rank's slot (reduce-scatter
  half), then ``k_p2p_rs_reduce`` (owner sum + broadcast + per-CTA cross-rank barrier);
* ``fused_rs``  -- the first of those two kernels only (the reduce-scatter half);
* ``nccl``      -- the GEMM into a local buffer, NCCL all-reduce, add.

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 -m fak_b200.benchmarks.rsbench \\
        --m 1280 --n 3584 --k 1792
"""
from __future__ import annotations

import argparse
import json
import os

import torch


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--m", type=int, default=1280)
    ap.add_argument("--n", type=int, default=3584)
    ap.add_argument("--k", type=int, default=0, help="this rank's K slice (default 3584 / world)")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--variants", default="gemm,fused_rs,fused,nccl")
    args = ap.parse_args(argv)
    import torch.distributed as dist

    from fak_b200.ops._ext import ext
    from fak_b200.parallel import dist as pdist
    from fak_b200.parallel.p2p import MAX_CTAS, MAX_W, RS_CTAS, PeerBuffer, _align

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = pdist.init(world, rank, local)
    M, N = args.m, args.n
    Kc = args.k or 3584 // world
    g = torch.Generator(device=dev).manual_seed(11 + rank)
    a = (torch.randn(M, Kc, device=dev, generator=g) * 0.1).bfloat16()
    w = (torch.randn(N, Kc, device=dev, generator=g) * 0.02).bfloat16()
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    # peer buffer: barrier flags [1 site][MAX_CTAS][MAX_W], residual x [M, N], partial slots
    # [W][MR][N] (MR rows of owned 128-row m-blocks), tile flags [m-block][256-column block][MAX_W]
    n_m, n_n = -(-M // 128), -(-N // 256)
    MR = -(-n_m // world) * 128
    off = 0
    bar_off = off
    off = _align(off + MAX_CTAS * MAX_W * 4)
    x_off = off
    off = _align(off + M * N * 4)
    parts_off = off
    off = _align(off + world * MR * N * 4)
    flags_off = off
    off = _align(off + n_m * n_n * MAX_W * 4)
    mem = PeerBuffer(off, group, dev)
    peers = torch.tensor(mem.ptrs, dtype=torch.int64)
    counters = torch.zeros(MAX_CTAS, dtype=torch.int32, device=dev)
    x = mem.buf[x_off:x_off + M * N * 4].view(torch.float32).view(M, N)
    part = torch.zeros(M, N, device=dev)
    epoch = [0]

    def one(v: str) -> None:
        if v == "gemm":
            ext().gemm_bf16(a, w, part, None, 0, err)
        elif v in ("fused", "fused_rs"):
            epoch[0] += 1
            ext().gemm_bf16_rs(a, w, peers, rank, parts_off, flags_off, MR, epoch[0], err)
            if v == "fused":
                ext().p2p_rs_reduce(peers, parts_off, flags_off, x_off, M, N, MR, rank, epoch[0], bar_off, 0,
                                    counters, err, RS_CTAS, 0)
        else:
            ext().gemm_bf16(a, w, part, None, 0, err)
            dist.all_reduce(part, group=group)
            x.add_(part)

    flops = 2.0 * M * N * Kc
    out = {"bench": "rsbench", "n_gpus": world, "m": M, "n": N, "k_per_rank": Kc,
           "nvlink_bytes_per_rank_out": round(2 * (world - 1) / world * M * N * 4 / 1e6, 2),
           "us_max_over_ranks": {}, "gemm_tflops": None}
    for v in args.variants.split(","):
        for _ in range(3):
            one(v)
        torch.cuda.synchronize()
        dist.barrier(group=group)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.iters):
            one(v)
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) * 1e3 / args.iters], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        out["us_max_over_ranks"][v] = round(float(t), 2)
        if v == "gemm":
            out["gemm_tflops"] = round(flops / float(t) / 1e6, 1)
        dist.barrier(group=group)
    out["error_word"] = int(err.item())
    if rank == 0:
        print(json.dumps(out), flush=True)
    mem.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
