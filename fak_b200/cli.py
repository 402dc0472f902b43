"""Command line: ``python -m fak_b200 <command>``.

  serve    run the gateway over a local model (GGUF file or a synthetic preset) or an upstream
           OpenAI-compatible server (reference: cmd/fak/serve.go:131-183)
  guard    wrap an agent command behind the gateway: the agent's OpenAI/Anthropic base URLs
           point at the floor, every tool call it is offered is adjudicated and journaled
           (reference: cmd/fak/guard.go:101-160, ``--gguf`` runs the model in-process)
  synth    write a random-init GGUF checkpoint of a named architecture
  inspect  print a GGUF file's metadata and tensor directory
  adjudicate  run one tool call (JSON) through a policy and print the verdict
"""
from __future__ import annotations

import argparse
import json
import os
import socket
import subprocess
import sys
import threading
import time


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def build_gateway(args):
    from .agentkernel import Kernel, default_policy, load_policy
    from .serve import Gateway
    policy = load_policy(args.policy) if getattr(args, "policy", None) else default_policy()
    kernel = Kernel(policy, journal_path=getattr(args, "journal", None))
    if getattr(args, "upstream", None):
        from .serve import UpstreamBackend
        backend = UpstreamBackend(args.upstream, os.environ.get("FAK_UPSTREAM_API_KEY", ""))
    else:
        backend = build_model_backend(args)
    return Gateway(backend, kernel, model_name=args.model_name,
                   ctx_view_budget=getattr(args, "ctx_view_budget", 0))


def build_model_backend(args):
    from .config import EngineConfig, preset
    from .gguf import open_gguf
    from .tokenizer import Tokenizer
    hf = getattr(args, "hf", None)
    if args.cpu:
        from .models.reference import ReferenceModel
        from .serve import ReferenceBackend
        if hf:
            import json
            with open(os.path.join(hf, "config.json")) as f:
                mt = str(json.load(f).get("model_type", ""))
            if mt == "glm_moe_dsa" or mt.startswith("gemma4"):   # whole-sequence models
                from .serve.backend import CachelessModel
                if mt == "glm_moe_dsa":
                    from .models.glm_dsa import GlmDsaReference as whole
                else:
                    from .models.gemma4 import Gemma4Reference as whole
                ref = CachelessModel(whole.from_hf(hf))
            else:
                from .models.hf import load_reference_tensors_hf
                cfg, tensors = load_reference_tensors_hf(hf)
                ref = ReferenceModel(cfg, tensors)
            tok = Tokenizer.from_tokenizer_json(os.path.join(hf, "tokenizer.json"))
        elif args.gguf:
            ref = ReferenceModel.from_gguf(args.gguf)
            tok = Tokenizer.from_gguf_metadata(open_gguf(args.gguf).metadata)
        else:
            raise SystemExit("--cpu needs --gguf or --hf")
        if args.lora and not isinstance(ref, ReferenceModel):
            raise SystemExit("--lora needs a model that runs on the incremental reference forward")
        if args.lora:   # applied dynamically after each patched projection
            from .models.lora import LoRASet, load_peft_adapter
            ls = LoRASet()
            for d in args.lora:
                load_peft_adapter(d, ls)
            ref.set_lora(ls)
        return ReferenceBackend(ref, tok)
    import torch
    from .engine import Engine
    from .serve import EngineBackend
    ecfg = EngineConfig.from_env(max_batch=args.max_batch)
    if getattr(args, "cpu_offload_experts", False):
        ecfg.cpu_offload_experts = True
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    if hf:
        eng = Engine.from_hf(hf, ecfg, dev, max_context=args.max_context, lora=args.lora)
        tok = Tokenizer.from_tokenizer_json(os.path.join(hf, "tokenizer.json"))
    elif args.gguf:
        eng = Engine.from_gguf(args.gguf, ecfg, dev, max_context=args.max_context, lora=args.lora)
        tok = Tokenizer.from_gguf_metadata(open_gguf(args.gguf).metadata)
    else:
        import tempfile
        from .gguf.synth import write_metadata
        from .gguf.writer import GGUFWriter
        cfg = preset(args.synthetic)
        eng = Engine.synthetic(cfg, args.mix, 0, ecfg, dev, max_context=args.max_context)
        # vocabulary of the synthetic checkpoint (no weights needed for the tokenizer)
        path = os.path.join(tempfile.mkdtemp(), "vocab.gguf")
        w = GGUFWriter(path, arch=cfg.arch)
        write_metadata(w, cfg, args.mix)
        w.write()
        tok = Tokenizer.from_gguf_metadata(open_gguf(path).metadata)
    eng.warmup_graphs()
    return EngineBackend(eng, tok, name=args.model_name or "fak-b200")


def _add_model_args(ap):
    ap.add_argument("--gguf", help="GGUF checkpoint (Q4_K/Q6_K/Q8_0/f16/f32 blocks)")
    ap.add_argument("--hf", help="Hugging Face checkpoint directory (config.json, *.safetensors, tokenizer.json); "
                                 "float weights are quantized to Q8_0 on load")
    ap.add_argument("--lora", action="append", default=[],
                    help="PEFT LoRA adapter directory (repeatable; merged into the device weights at load)")
    ap.add_argument("--synthetic", default="tiny-qwen2", help="random-init preset when no --gguf is given")
    ap.add_argument("--mix", default="q4_k_m")
    ap.add_argument("--cpu", action="store_true", help="fp32 reference forward on the CPU")
    ap.add_argument("--upstream", help="proxy to an upstream OpenAI-compatible server instead of a local model")
    ap.add_argument("--policy", help="policy manifest (fak-policy/v1 JSON); default: built-in floor")
    ap.add_argument("--journal", help="append the hash-chained decision journal to this file")
    ap.add_argument("--model-name", default=None)
    ap.add_argument("--ctx-view-budget", type=int, default=0,
                    help="plan each chat prompt as a view of at most this many tokens (0: whole transcript)")
    ap.add_argument("--max-batch", type=int, default=32)
    ap.add_argument("--max-context", type=int, default=8192)
    ap.add_argument("--cpu-offload-experts", action="store_true",
                    help="keep MoE expert weights in host memory and run their FFNs on the CPU")


def cmd_serve(args) -> int:
    import uvicorn
    from .serve import create_app
    gw = build_gateway(args)
    uvicorn.run(create_app(gw), host=args.host, port=args.port, log_level="warning")
    return 0


def cmd_guard(args) -> int:
    import uvicorn
    from .serve import create_app
    if not args.command:
        raise SystemExit("usage: guard [options] -- <agent command ...>")
    gw = build_gateway(args)
    port = args.port or _free_port()
    server = uvicorn.Server(uvicorn.Config(create_app(gw), host="127.0.0.1", port=port, log_level="warning"))
    th = threading.Thread(target=server.run, daemon=True)
    th.start()
    for _ in range(200):
        if server.started:
            break
        time.sleep(0.05)
    env = dict(os.environ)
    env.update({"OPENAI_BASE_URL": f"http://127.0.0.1:{port}/v1", "OPENAI_API_BASE": f"http://127.0.0.1:{port}/v1",
                "ANTHROPIC_BASE_URL": f"http://127.0.0.1:{port}", "FAK_GATEWAY_URL": f"http://127.0.0.1:{port}"})
    cmd = args.command[1:] if args.command[0] == "--" else args.command
    rc = subprocess.call(cmd, env=env)
    server.should_exit = True
    th.join(timeout=5)
    ok, bad = gw.kernel.journal.verify()
    st = gw.kernel.stats
    print(json.dumps({"agent_exit": rc, "tool_calls": st["calls"], "allowed": st["allow"] + st["transform"],
                      "denied": st["deny"], "journal_chain_ok": ok}), file=sys.stderr)
    return rc


def cmd_synth(args) -> int:
    from .config import preset
    from .gguf.synth import write_synthetic_gguf
    write_synthetic_gguf(args.out, preset(args.preset), args.mix, args.seed, args.std,
                         device="cuda" if args.gpu else "cpu")
    print(args.out)
    return 0


def cmd_inspect(args) -> int:
    from .config import config_from_gguf_metadata
    from .gguf import open_gguf
    g = open_gguf(args.path)
    meta = {k: (v if not isinstance(v, list) or len(v) < 8 else f"[{len(v)} items]") for k, v in g.metadata.items()}
    cfg = config_from_gguf_metadata(g.metadata, {k: v.shape for k, v in g.tensors.items()})
    types: dict[str, int] = {}
    for t in g:
        types[t.ggml_type.name] = types.get(t.ggml_type.name, 0) + t.nbytes
    print(json.dumps({"config": cfg.__dict__, "bytes_by_type": types, "tensors": len(g.tensors), "metadata": meta},
                     indent=1, default=str))
    return 0


def cmd_adjudicate(args) -> int:
    from .agentkernel import Adjudicator, ToolCall, default_policy, load_policy
    a = Adjudicator(load_policy(args.policy) if args.policy else default_policy())
    v = a.adjudicate(ToolCall.from_dict(json.loads(args.call)))
    print(json.dumps(v.to_dict()))
    return 0 if v.allowed else 3


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="fak_b200")
    sub = ap.add_subparsers(dest="cmd", required=True)
    s = sub.add_parser("serve", help="run the gateway")
    _add_model_args(s)
    s.add_argument("--host", default="127.0.0.1")
    s.add_argument("--port", type=int, default=8080)
    s.set_defaults(fn=cmd_serve)
    g = sub.add_parser("guard", help="wrap an agent command behind the gateway")
    _add_model_args(g)
    g.add_argument("--port", type=int, default=0)
    g.add_argument("command", nargs=argparse.REMAINDER)
    g.set_defaults(fn=cmd_guard)
    y = sub.add_parser("synth", help="write a random-init GGUF")
    y.add_argument("preset")
    y.add_argument("out")
    y.add_argument("--mix", default="q8_0")
    y.add_argument("--seed", type=int, default=0)
    y.add_argument("--std", type=float, default=0.02)
    y.add_argument("--gpu", action="store_true")
    y.set_defaults(fn=cmd_synth)
    i = sub.add_parser("inspect", help="describe a GGUF file")
    i.add_argument("path")
    i.set_defaults(fn=cmd_inspect)
    d = sub.add_parser("adjudicate", help="adjudicate one tool call")
    d.add_argument("call", help='JSON, e.g. {"tool": "Bash", "args": {"command": "ls"}}')
    d.add_argument("--policy")
    d.set_defaults(fn=cmd_adjudicate)
    args = ap.parse_args(argv)
    return args.fn(args)


if __name__ == "__main__":
    sys.exit(main())
