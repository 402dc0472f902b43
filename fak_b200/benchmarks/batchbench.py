"""Aggregate decode throughput against the batch size (reference: cmd/batchbench).

Runs the model runner's graphed decode step at each batch size of ``--batches`` over contexts of
``--ctx`` tokens and prints one JSON line per batch (ms per step, tokens/s, weight-streaming
bandwidth in GB/s), then a summary line with the batch that maximises tokens/s.

    python -m fak_b200.benchmarks.batchbench --model qwen2.5-7b --batches 1,2,4,8,16,32,64 --ctx 2048
"""
from __future__ import annotations

import argparse
import json


def main(argv=None) -> list[dict]:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--model", default="qwen2.5-7b")
    ap.add_argument("--mix", default="q4_k_m")
    ap.add_argument("--batches", default="1,2,4,8,16,32")
    ap.add_argument("--ctx", type=int, default=2048)
    ap.add_argument("--steps", type=int, default=20)
    args = ap.parse_args(argv)
    from .modelbench import main as modelbench
    rows = []
    for b in (int(x) for x in args.batches.split(",")):
        r = modelbench(["--model", args.model, "--mix", args.mix, "--batch", str(b), "--ctx", str(args.ctx),
                        "--steps", str(args.steps), "--decode-only"])
        r["weight_gb_s"] = round(r["weight_bytes"] / (r["decode_ms_per_step"] * 1e6), 1)
        rows.append(r)
    best = max(rows, key=lambda r: r["decode_tok_s"])
    print(json.dumps({"summary": True, "best_batch": best["batch"], "best_tok_s": best["decode_tok_s"],
                      "tok_s_by_batch": {r["batch"]: r["decode_tok_s"] for r in rows}}), flush=True)
    return rows


if __name__ == "__main__":
    main()
