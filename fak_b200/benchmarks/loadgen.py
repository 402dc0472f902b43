"""Concurrency sweep against an OpenAI-compatible chat endpoint (a fak-b200 gateway or any server).

For each concurrency level C, C client threads issue streamed chat completions back to back for a
fixed number of requests; per request the time to the first content delta (TTFT), the mean time
between later deltas (TPOT) and the delta count are recorded.  One JSON line per level: request
rate, delta throughput, p50 / p90 / p99 TTFT and TPOT.

    python -m fak_b200.benchmarks.loadgen --url http://127.0.0.1:8000 --concurrency 1,4,16 --requests 32

Reference: cmd/loadgen (OpenAI endpoint concurrency sweep).
"""
from __future__ import annotations

import argparse
import json
import threading
import time

import numpy as np

from ..client import FakClient


def _pct(xs, q):
    return float(np.percentile(xs, q)) if xs else None


def run_level(make_client, concurrency: int, n_requests: int, prompt: str, max_tokens: int) -> dict:
    lock = threading.Lock()
    todo = list(range(n_requests))
    ttft, tpot, deltas, errors = [], [], [], []

    def worker():
        c = make_client()
        while True:
            with lock:
                if not todo:
                    return
                i = todo.pop()
            t0 = time.perf_counter()
            first, last, n = None, None, 0
            try:
                for _ in c.stream_chat([{"role": "user", "content": f"{prompt} #{i}"}], max_tokens=max_tokens):
                    now = time.perf_counter()
                    if first is None:
                        first = now
                    last = now
                    n += 1
            except Exception as e:   # recorded, the sweep goes on
                with lock:
                    errors.append(repr(e)[:200])
                continue
            with lock:
                deltas.append(n)
                if first is not None:
                    ttft.append(first - t0)
                    if n > 1:
                        tpot.append((last - first) / (n - 1))

    t0 = time.perf_counter()
    threads = [threading.Thread(target=worker) for _ in range(concurrency)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    wall = time.perf_counter() - t0
    ms = lambda v: None if v is None else round(1000 * v, 3)
    return {"concurrency": concurrency, "requests": len(deltas), "errors": len(errors), "wall_s": round(wall, 3),
            "req_per_s": round(len(deltas) / wall, 3), "deltas_per_s": round(sum(deltas) / wall, 2),
            "ttft_ms_p50": ms(_pct(ttft, 50)), "ttft_ms_p90": ms(_pct(ttft, 90)), "ttft_ms_p99": ms(_pct(ttft, 99)),
            "tpot_ms_p50": ms(_pct(tpot, 50)), "tpot_ms_p90": ms(_pct(tpot, 90)),
            "first_error": errors[0] if errors else None}


def main(argv=None) -> list[dict]:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--url", default="http://127.0.0.1:8000")
    ap.add_argument("--api-key", default="")
    ap.add_argument("--concurrency", default="1,4,16")
    ap.add_argument("--requests", type=int, default=32)
    ap.add_argument("--max-tokens", type=int, default=64)
    ap.add_argument("--prompt", default="Summarise the plan in one paragraph.")
    args = ap.parse_args(argv)
    out = []
    for c in (int(x) for x in args.concurrency.split(",")):
        r = run_level(lambda: FakClient(args.url, args.api_key), c, args.requests, args.prompt, args.max_tokens)
        print(json.dumps(r), flush=True)
        out.append(r)
    return out


if __name__ == "__main__":
    main()
