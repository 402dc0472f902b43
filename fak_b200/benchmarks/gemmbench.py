"""tcgen05 bf16 GEMM benchmark (the prefill linear layers): out[M, N] = a[M, K] . W[N, K]^T.

    python -m fak_b200.benchmarks.gemmbench --m 1280 --n 37888 --k 3584
"""
from __future__ import annotations

import argparse
import json

import torch


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--m", type=int, default=1280)
    ap.add_argument("--n", type=int, default=37888)
    ap.add_argument("--k", type=int, default=3584)
    ap.add_argument("--epi", type=int, default=0, help="0 store, 1 add, 2 SwiGLU")
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args(argv)
    from fak_b200.ops._ext import ext

    dev = torch.device("cuda", 0)
    a = torch.randn(args.m, args.k, device=dev).bfloat16()
    # two weight copies so consecutive launches do not find the weights in L2
    ws = [torch.randn(args.n, args.k, device=dev).bfloat16() for _ in range(2)]
    out = torch.zeros(args.m, args.n // 2 if args.epi == 2 else args.n, device=dev)
    C = ext()
    for i in range(3):
        C.gemm_bf16(a, ws[i % 2], out, None, args.epi, None)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.iters):
        C.gemm_bf16(a, ws[i % 2], out, None, args.epi, None)
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000 / args.iters
    flops = 2.0 * args.m * args.n * args.k
    print(json.dumps({"kernel": "gemm_bf16 (tcgen05)", "m": args.m, "n": args.n, "k": args.k, "epi": args.epi,
                      "us": round(us, 2), "tflops": round(flops / us / 1e6, 1)}))


if __name__ == "__main__":
    main()
