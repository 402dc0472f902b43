"""Paged decode-attention benchmark: B sequences x ctx tokens over 16-token pages (CUDA events).

Builds ``--layers`` independent KV caches (so consecutive launches stream from DRAM rather than
L2), optionally sharing the first ``--shared`` tokens' pages between all sequences as the radix
cache does, and times split-KV decode attention plus its combine.  Reports the KV bytes each launch
must read (shared pages counted once) and the effective bandwidth.

    python -m fak_b200.benchmarks.attnbench --batch 5 --ctx 9000 --shared 8192
    python -m fak_b200.benchmarks.attnbench --batch 8 --ctx 4096 --shared 0 --prefill 4096 --impl tc
"""
from __future__ import annotations

import argparse
import json
import math

import torch


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=5)
    ap.add_argument("--ctx", type=int, default=9000)
    ap.add_argument("--shared", type=int, default=8192, help="leading tokens whose pages all sequences share")
    ap.add_argument("--heads", type=int, default=28)
    ap.add_argument("--kv-heads", type=int, default=4)
    ap.add_argument("--head-dim", type=int, default=128)
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--split", type=int, default=16)
    ap.add_argument("--pps", type=int, default=1, help="pages per split (a lower bound; with --split large enough "
                    "for the context, each split holds exactly this many pages)")
    ap.add_argument("--prefill", type=int, default=0,
                    help="time prefill attention instead: each sequence's last N tokens attend to the whole context")
    ap.add_argument("--impl", default="tc", choices=("tc", "fa2"),
                    help="prefill kernel: tcgen05 / TMEM (head dim 128) or the mma.sync one")
    ap.add_argument("--cascade", type=int, default=0,
                    help="prefix splits of cascade attention over the shared pages (0: plain split-KV path)")
    args = ap.parse_args(argv)
    from fak_b200.ops import kernels as K

    dev = torch.device("cuda", 0)
    B, H, Hkv, D, ctx = args.batch, args.heads, args.kv_heads, args.head_dim, args.ctx
    n_sh = min(args.shared, ctx) // 16
    per_seq = math.ceil(ctx / 16)
    n_pages = n_sh + B * (per_seq - n_sh) + 1
    g = torch.Generator(device=dev).manual_seed(0)
    k_all = torch.randn(args.layers, n_pages, Hkv, 16, D, device=dev, generator=g).bfloat16()
    v_all = torch.randn(args.layers, n_pages, Hkv, 16, D, device=dev, generator=g).bfloat16()
    caches = [(k_all[i], v_all[i]) for i in range(args.layers)]
    bt = torch.zeros(B, per_seq, dtype=torch.int32)
    nxt = 1 + n_sh
    for b in range(B):
        bt[b, :n_sh] = torch.arange(1, 1 + n_sh)
        bt[b, n_sh:] = torch.arange(nxt, nxt + per_seq - n_sh)
        nxt += per_seq - n_sh
    bt = bt.to(dev)
    ctx_t = torch.full((B,), ctx, dtype=torch.int32, device=dev)
    q = torch.randn(B, H, D, device=dev)
    act = K.ActQ(B, H * D, dev)
    ws = torch.zeros(B * H * (args.split + args.cascade) * (D + 2), device=dev)
    shared = torch.tensor([n_sh], dtype=torch.int32, device=dev)
    casc = {"shared_pages": shared, "prefix_splits": args.cascade} if args.cascade else {}

    def run(i):
        kc, vc = caches[i % args.layers]
        K.decode_attention(q, kc, vc, bt, ctx_t, args.split, act=act, workspace=ws, pages_per_split=args.pps, **casc)

    if args.prefill:   # B chunks of the last `prefill` tokens over the cached context
        from fak_b200.models.runner import PrefillMeta
        Q = args.prefill
        meta = PrefillMeta.build([Q] * B, [ctx - Q] * B, dev)
        qp = torch.randn(B * Q, H, D, device=dev, generator=g).bfloat16()
        outp = torch.empty(B * Q, H * D, device=dev, dtype=torch.bfloat16)

        def run(i):  # noqa: F811
            if args.impl == "tc":
                K.prefill_attention_tc(qp, k_all, v_all, i % args.layers, bt, meta, outp)
            else:
                kc, vc = caches[i % args.layers]
                K.prefill_attention(qp, kc, vc, bt, meta, outp)

    for i in range(3):
        run(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.iters):
        run(i)
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000 / args.iters
    page_bytes = 2 * Hkv * 16 * D * 2
    unique = (n_sh + B * (per_seq - n_sh)) * page_bytes
    extra = {}
    if args.prefill:   # causal QK^T and PV FLOPs: query j of a chunk sees ctx - Q + j + 1 keys
        Q = args.prefill
        keys = B * (Q * (ctx - Q) + Q * (Q + 1) // 2)
        flops = 4 * D * H * keys
        extra = {"impl": args.impl, "tflops": round(flops / us / 1e6, 1)}
    print(json.dumps({"kernel": "prefill_attention" if args.prefill else "decode_attention+combine",
                      "prefill": args.prefill, **extra,
                      "batch": B, "ctx": ctx, "shared": n_sh * 16,
                      "heads": H, "kv_heads": Hkv, "head_dim": D, "splits": args.split, "pps": args.pps,
                      "cascade": args.cascade,
                      "us": round(us, 2),
                      "unique_kv_bytes": unique, "tb_s_unique": round(unique / us / 1e6, 3),
                      "tb_s_streamed": round(B * per_seq * page_bytes / us / 1e6, 3)}))


if __name__ == "__main__":
    main()
