"""GPU engine against the C++ CPU runtime on one checkpoint (reference: cmd/gpucheck -- a real
model's GPU greedy continuation must agree with the CPU path).

Both runs read the same GGUF (a given file, or a seeded synthetic one of ``--preset``): the CPU
runtime steps the prompt token by token, the engine prefills it and decodes greedily.  Reported:
cosine of the prompt's last logits, the agreeing prefix of the greedy continuations, and the
teacher-forced argmax agreement (the CPU logits of every step are compared with the engine's
logits on the same forced tokens).  One JSON line; ``ok`` when the logits agree (cosine >=
``--min-cos``) and the continuations agree on at least ``--min-prefix`` tokens (int8 activations on
both sides round differently, so a near-tie may flip a later token).

    python -m fak_b200.benchmarks.gpucheck --preset smollm2-135m --mix q8_0 --prompt 64 --new 32
"""
from __future__ import annotations

import argparse
import json
import os
import tempfile

import numpy as np
import torch


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gguf", default="", help="checkpoint (default: a synthetic one of --preset)")
    ap.add_argument("--preset", default="smollm2-135m")
    ap.add_argument("--mix", default="q8_0")
    ap.add_argument("--prompt", type=int, default=64)
    ap.add_argument("--new", type=int, default=32)
    ap.add_argument("--min-cos", type=float, default=0.99)
    ap.add_argument("--min-prefix", type=int, default=8)
    args = ap.parse_args(argv)
    from fak_b200.config import EngineConfig, preset
    from fak_b200.engine import Engine
    from fak_b200.gguf.synth import write_synthetic_gguf
    from fak_b200.models.cpu import load_cpu_model
    path = args.gguf
    if not path:
        path = os.path.join(tempfile.mkdtemp(), f"{args.preset}.gguf")
        write_synthetic_gguf(path, preset(args.preset), args.mix, seed=0)
    cpu, cfg = load_cpu_model(path, act_quant=True)
    prompt = np.random.default_rng(0).integers(0, cfg.vocab_size, args.prompt).tolist()
    cpu.reset()
    for t in prompt:
        lg = np.asarray(cpu.step(t), dtype=np.float32)
    first_cpu = lg.copy()
    cpu_out = []
    for _ in range(args.new):
        nxt = int(np.argmax(lg))
        cpu_out.append(nxt)
        lg = np.asarray(cpu.step(nxt), dtype=np.float32)

    dev = torch.device("cuda", 0)
    eng = Engine.from_gguf(path, EngineConfig(max_batch=4, kv_pages=512, cuda_graph=True, graph_batch_buckets=(1,)),
                           dev, max_context=max(2048, args.prompt + args.new + 32))
    eng.warmup_graphs()
    from fak_b200.benchmarks.tpcheck import forced_logits
    gl = forced_logits(eng, prompt, cpu_out[:-1])               # [1 + new - 1, V]: the prompt's, then forced
    gpu_out = eng.generate([prompt], args.new)[0]
    eng.shutdown()
    # CPU logits on the same forced tokens
    cpu.reset()
    rows = []
    for t in prompt:
        lg = np.asarray(cpu.step(t), dtype=np.float32)
    rows.append(lg)
    for t in cpu_out[:-1]:
        rows.append(np.asarray(cpu.step(t), dtype=np.float32))
    cl = torch.from_numpy(np.stack(rows))[:, :cfg.vocab_size]
    gl = gl[:, :cfg.vocab_size]
    cos = torch.nn.functional.cosine_similarity(gl, cl, dim=1)
    first_cos = float(torch.nn.functional.cosine_similarity(gl[0], torch.from_numpy(first_cpu[:cfg.vocab_size]),
                                                            dim=0))
    k = 0
    while k < len(gpu_out) and gpu_out[k] == cpu_out[k]:
        k += 1
    agree = float((gl.argmax(1) == cl.argmax(1)).float().mean())
    ok = first_cos >= args.min_cos and float(cos.min()) >= args.min_cos and k >= min(args.min_prefix, args.new)
    print(json.dumps({"bench": "gpucheck", "model": cfg.name, "mix": args.mix, "prompt": args.prompt, "new": args.new,
                      "first_logits_cos": round(first_cos, 6), "min_step_cos": round(float(cos.min()), 6),
                      "teacher_forced_argmax_agreement": round(agree, 4), "greedy_prefix": k,
                      "gpu_first": gpu_out[:8], "cpu_first": cpu_out[:8], "ok": ok}), flush=True)
    return 0 if ok else 1


if __name__ == "__main__":
    raise SystemExit(main())
