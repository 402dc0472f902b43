"""CPU-path benchmark: SmolLM2-135M architecture, random-init N(0, 0.02)
weights written as GGUF Q8_0, greedy decode of 128 tokens after a 256-token seeded prompt, batch 1,
through the C++ CPU runtime.

    python -m fak_b200.benchmarks.cpubench [--preset smollm2-135m] [--prompt 256] [--new 128]
"""
from __future__ import annotations

import argparse
import json
import os
import tempfile
import time

import numpy as np


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--preset", default="smollm2-135m")
    ap.add_argument("--mix", default="q8_0")
    ap.add_argument("--prompt", type=int, default=256)
    ap.add_argument("--new", type=int, default=128)
    ap.add_argument("--fp32-oracle", action="store_true", help="dequantize to fp32 instead of int8 activations")
    args = ap.parse_args(argv)
    from fak_b200.config import preset
    from fak_b200.gguf.synth import write_synthetic_gguf
    from fak_b200.models.cpu import load_cpu_model
    cfg = preset(args.preset)
    path = os.path.join(tempfile.mkdtemp(), f"{args.preset}.gguf")
    write_synthetic_gguf(path, cfg, args.mix, seed=0)
    m, _ = load_cpu_model(path, act_quant=not args.fp32_oracle)
    prompt = np.random.default_rng(0).integers(0, cfg.vocab_size, args.prompt).tolist()
    t0 = time.perf_counter()
    m.reset()
    for t in prompt:
        lg = m.step(t)
    t1 = time.perf_counter()
    out = []
    for i in range(args.new):
        nxt = int(np.argmax(lg))
        out.append(nxt)
        lg = m.step(nxt)
    t2 = time.perf_counter()
    print(json.dumps({"preset": args.preset, "mix": args.mix, "threads": m.threads(), "prompt": args.prompt,
                      "new": args.new, "prefill_tok_s": round(args.prompt / (t1 - t0), 1),
                      "decode_tok_s": round(args.new / (t2 - t1), 1), "first_tokens": out[:8]}))


if __name__ == "__main__":
    main()
