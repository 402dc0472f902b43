"""Bandwidth of the quantized decode GEMV kernels (tile-packed tgemv, row-major qmmv / qgemv) on one weight matrix (CUDA events, L2 > working set).

    python -m fak_b200.benchmarks.gemvbench --rows 37888 --cols 3584 --qtype 12 --batch 5
    python -m fak_b200.benchmarks.gemvbench --rows 4096 --cols 3584 --qtype 12 --pair-rows 512 --unit 1
"""
from __future__ import annotations

import argparse
import json

import torch


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=37888)
    ap.add_argument("--cols", type=int, default=3584)
    ap.add_argument("--qtype", type=int, default=12)
    ap.add_argument("--batch", type=int, default=5)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--kernel", default="tgemv", choices=["tgemv", "qmmv", "qgemv"])
    ap.add_argument("--flags", type=int, default=0)
    ap.add_argument("--unit", type=int, default=0, help="1: activations with one scale per 256 columns")
    ap.add_argument("--pair-rows", type=int, default=0,
                    help="also a Q6_K matrix of this many rows over the same activations, both in one pair launch")
    ap.add_argument("--graph", type=int, default=1, help="1: time the launches replayed from a CUDA graph "
                    "(device time per launch; 0: eager launches, host-bound for small matrices)")
    args = ap.parse_args(argv)
    from fak_b200.models.weights import QuantWeight
    from fak_b200.ops import kernels as K
    from fak_b200.ops import quant as dq
    from fak_b200.ops._ext import ext
    dev = torch.device("cuda", 0)
    # several copies so consecutive launches stream from DRAM, not L2 (126 MB)
    n_copies = max(2, int(400e6 // (args.rows * dq.row_bytes(args.qtype, args.cols))) + 1)
    ws = []
    for i in range(n_copies):
        raw = dq.synth_quantized((args.rows, args.cols), args.qtype, 1234 + i, 0.02, device="cuda")
        w = QuantWeight.from_rows(raw.view(args.rows, -1), args.qtype, args.cols, dev)
        if args.kernel == "tgemv":
            w.pack()
            w.buf = None  # only the tile-packed copy is streamed
        ws.append(w)
    wbs = []
    if args.pair_rows:
        assert args.kernel == "tgemv" and args.qtype == 12, "the pair launch takes a Q4_K matrix first"
        for i in range(n_copies):
            raw = dq.synth_quantized((args.pair_rows, args.cols), 14, 4321 + i, 0.02, device="cuda")
            wb = QuantWeight.from_rows(raw.view(args.pair_rows, -1), 14, args.cols, dev).pack()
            wb.buf = None
            wbs.append(wb)
    act = K.ActQ(max(8, args.batch), args.cols, dev, unit=bool(args.unit))
    K.quant_act(torch.randn(args.batch, args.cols, device=dev), act)
    y = torch.zeros(max(8, args.batch), args.rows, device=dev)
    yb = torch.zeros(max(8, args.batch), max(1, args.pair_rows), device=dev)
    C = ext()

    part, cnt = K.tgemv_workspace(dev, ws + wbs)

    def run(w, i=0):
        if wbs:
            assert K.gemv_pair(w, wbs[i % n_copies], act, args.batch, y, yb)
        elif args.kernel == "tgemv":
            C.tgemv(w.tp, w.qtype, w.rows, w.cols, act.q, act.ds, None, None, 0.0, args.batch, y, None, 0, part, cnt,
                    None, args.flags, unit=act.unit)
        elif args.kernel == "qmmv":
            C.qmmv(w.buf, w.qtype, w.rows, w.cols, w.pitch, act.q, act.ds, args.batch, y, None, 0, args.flags)
        else:
            C.qgemv(w.buf, w.qtype, w.rows, w.cols, w.pitch, act.q, act.ds, args.batch, y, None, 0)
    for i in range(3):
        run(ws[i % n_copies], i)
    torch.cuda.synchronize()
    g = None
    if args.graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(args.iters):
                run(ws[i % n_copies], i)
        g.replay()
        torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    if g is not None:
        g.replay()
    else:
        for i in range(args.iters):
            run(ws[i % n_copies], i)
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000 / args.iters
    nbytes = ws[0].nbytes + (wbs[0].nbytes if wbs else 0)
    info = {}
    if args.kernel == "tgemv":
        S, ticket, slices, W, R, smem = C.tgemv_workspace(args.qtype, args.rows, args.cols, 0)
        info = {"slices": slices, "warps": W, "depth": R, "smem": smem}
    print(json.dumps({"kernel": args.kernel, **info, "rows": args.rows, "cols": args.cols, "qtype": args.qtype,
                      "pair_rows": args.pair_rows, "graph": bool(args.graph),
                      "batch": args.batch, "flags": args.flags, "unit": act.unit, "us": round(us, 2),
                      "tb_s": round(nbytes / us / 1e6, 3)}))


if __name__ == "__main__":
    main()
