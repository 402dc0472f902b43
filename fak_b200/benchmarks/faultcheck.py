"""Failure detection on the fused tensor-parallel path: a peer that never arrives.

Two ranks (torchrun, one GPU each; run with NCCL_NVLS_ENABLE=0) build the same tiny TP=2 engine with a
short cross-rank spin limit and peer buffers mapped through CUDA IPC (no multicast object).  Both
prefill a request together (NCCL) and decode a few tokens normally.  Then rank 1 stays idle between
steps -- it launches nothing more and waits on a host-side (gloo) barrier -- while rank 0 keeps
decoding: its fused o_proj / down all-reduce waits for rank 1's tile flags, which nothing sets, gives
up after the spin limit, records error 4 in the step's kernel error word (the distributed argmax's
barrier records 1 in the collective word) and returns.  The engine reads the words back with the
step's tokens and raises DeviceStepError instead of emitting tokens.  Rank 0 then checks that its
CUDA context still works.  No GPU is faulted, trapped or hung: every wait is bounded.

    NCCL_NVLS_ENABLE=0 python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \\
        -m fak_b200.benchmarks.faultcheck
"""
from __future__ import annotations

import argparse
import json
import os
import time

import numpy as np
import torch
import torch.distributed as dist


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="tiny-qwen2")
    ap.add_argument("--spin", type=int, default=1 << 16, help="polls before a cross-rank wait gives up")
    args = ap.parse_args(argv)
    from fak_b200.config import EngineConfig, preset
    from fak_b200.engine import Engine
    from fak_b200.parallel import dist as pdist
    from fak_b200.parallel.errors import DeviceStepError
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != 2:
        raise SystemExit("faultcheck runs on exactly 2 ranks")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = pdist.init(world, rank, local, timeout_s=60)
    host = dist.new_group(backend="gloo")
    cfg = preset(args.model)
    ecfg = EngineConfig(max_batch=4, kv_pages=256, cuda_graph=True, graph_batch_buckets=(1,),
                        fused_collectives=True, p2p_spin_limit=args.spin)
    eng = Engine.synthetic(cfg, "q4_k_m", 3, ecfg, dev, max_context=512, tp_group=group, std=0.05)
    eng.warmup_graphs()
    prompt = np.random.default_rng(1).integers(0, cfg.vocab_size, 40).tolist()
    healthy = eng.generate([prompt], 6)[0]          # both ranks: a normal request
    r = eng.add_request(prompt, 64)
    eng._admit()
    eng._run_prefill()                                # both ranks: the prefill's NCCL collectives
    for _ in range(3):
        eng.step()                                    # both ranks: three fused decode steps
    torch.cuda.synchronize()
    res = {"rank": rank, "healthy_tokens": healthy}
    if rank == 0:
        t0 = time.perf_counter()
        err = None
        try:
            for _ in range(8):
                eng.step()                            # rank 1 launches nothing from here on
        except DeviceStepError as e:
            err = e
        res.update({"raised": err is not None, "seconds_to_error": round(time.perf_counter() - t0, 3),
                    "kernel_code": getattr(err, "kernel_code", None),
                    "collective_code": getattr(err, "collective_code", None),
                    "request_finish_reason": r.finish_reason})
        # the context is still usable after the expired waits
        x = torch.arange(1024, device=dev, dtype=torch.float32)
        res["context_ok"] = bool(float(x.sum().item()) == 1023 * 1024 / 2)
    dist.barrier(group=host)                          # rank 1 idles here, between steps
    box = [res]
    out = [None, None]
    dist.all_gather_object(out, box[0], group=host)
    if rank == 0:
        r0 = out[0]
        ok = (r0["raised"] and r0["kernel_code"] == 4 and r0["request_finish_reason"] == "error"
              and r0["context_ok"] and out[0]["healthy_tokens"] == out[1]["healthy_tokens"])
        print(json.dumps({"ranks": out, "ok": ok}), flush=True)
    # teardown: release graphs and unmap the peer buffers on both ranks; the NCCL communicator is
    # not used again (the ranks' collective epochs now differ)
    eng._pending = None
    eng.runner._graphs.clear()
    torch.cuda.synchronize()
    dist.barrier(group=host)
    if eng.runner.coll.mem is not None:
        mem = eng.runner.coll.mem
        mem.group = host                              # unmap in lockstep over the host group
        mem.close()
    dist.barrier(group=host)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
