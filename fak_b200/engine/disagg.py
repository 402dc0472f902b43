"""Prefill / decode disaggregation: prompts are prefilled on one engine and decoded on others.

* ``prefill_handoffs(engine, prompts)`` -- the prefill side: each prompt is prefilled (its prefix
  served from the radix cache when cached), the first token is sampled, and the prompt's K/V pages
  are exported as a ``KVHandoff`` (bf16 [layers, pages, kv heads, page, head dim] for K and V);
* ``adopt(engine, handoff, ...)`` -- the decode side: the request enters the engine with its K/V
  copied into freshly allocated pages (the swap-in path: device-to-device over NVLink when the
  handoff lives on another GPU, host-to-device from pinned memory otherwise) and continues
  decoding from the first token -- no recompute;
* ``send_handoff`` / ``recv_handoff`` -- the handoff between processes over torch.distributed
  point-to-point (NCCL over NVLink between GPUs, gloo between CPU processes): a fixed int64 header,
  the prompt ids, then K and V;
* ``PDCluster`` -- one prefill engine and N decode engines in one process; each handoff goes to the
  decode engine with the least work.

Reference: NativePDCluster (internal/modelengine/native_pd.go:233-520) and its KV transfer frames
(internal/model/paged_kv_transfer.go:26-327) over local / TCP transports.
"""
from __future__ import annotations

import dataclasses
import time

import torch
import torch.distributed as dist

from .sampling import SamplingParams

_HDR = 8   # prompt len, first token, layers, pages, kv heads, page size, head dim, dtype code
_DT = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}
_DT_INV = {v: k for k, v in _DT.items()}


@dataclasses.dataclass
class KVHandoff:
    prompt: list[int]
    first_token: int
    k: torch.Tensor     # [L, n_pages, Hkv, page, D]
    v: torch.Tensor
    page_size: int
    ttft_s: float = 0.0

    @property
    def nbytes(self) -> int:
        return 2 * self.k.numel() * self.k.element_size()


def prefill_handoffs(engine, prompts: list[list[int]], sampling: SamplingParams | None = None,
                     to_host: bool = False) -> list[KVHandoff]:
    """Prefill ``prompts`` on ``engine`` and export each one's K/V (kept on its device unless
    ``to_host``: then in pinned host memory)."""
    t0 = time.perf_counter()
    reqs = [engine.add_request(p, 1, sampling) for p in prompts]
    for r in reqs:
        r.hold_pages = True
    engine.run_until_done(reqs)
    out = []
    for r in reqs:
        idx = torch.tensor(r.held_pages, dtype=torch.long).to(engine.device, non_blocking=True)
        kv = []
        for t in (engine.kv.k, engine.kv.v):
            g = t.index_select(1, idx)
            if to_host:
                h = torch.empty(g.shape, dtype=g.dtype, pin_memory=True)
                h.copy_(g, non_blocking=True)
                g = h
            kv.append(g)
        engine.pool.release(r.held_pages)   # stream-ordered after the gathers above
        r.held_pages = []
        out.append(KVHandoff(list(r.prompt), r.output[0], kv[0], kv[1], engine.ecfg.page_size,
                             (r.first_token_time or time.perf_counter()) - t0))
    if to_host:
        torch.cuda.synchronize(engine.device)
    return out


def adopt(engine, h: KVHandoff, max_new_tokens: int, sampling: SamplingParams | None = None, stop_ids=(),
          on_token=None):
    """Continue a handed-over request on ``engine``; returns its Request (output starts with the
    handoff's first token)."""
    from .engine import Request
    if h.page_size != engine.ecfg.page_size:
        raise ValueError(f"handoff page size {h.page_size} != engine page size {engine.ecfg.page_size}")
    if tuple(h.k.shape[0:1] + h.k.shape[2:]) != (engine.kv.k.shape[0],) + tuple(engine.kv.k.shape[2:]):
        raise ValueError(f"handoff K/V {tuple(h.k.shape)} does not match the engine's cache {tuple(engine.kv.k.shape)}")
    if len(h.prompt) + max_new_tokens > engine.max_context:
        raise ValueError("prompt + new tokens exceed the decode engine's context")
    r = Request(next(engine._rid), list(h.prompt), max_new_tokens, sampling or SamplingParams(),
                frozenset(stop_ids), on_token=on_token)
    r.tokens = list(h.prompt)
    r.first_token_time = time.perf_counter()
    engine._emit(r, h.first_token)   # n_kv 0 and no pages yet: a request that ends here caches nothing
    if r.finished:
        return r
    r.n_kv = len(h.prompt)
    r.swap = (h.k, h.v, 0)
    engine.swapped.append(r)
    return r


def send_handoff(h: KVHandoff, dst: int, group=None) -> None:
    dev = h.k.device
    hdr = torch.tensor([len(h.prompt), h.first_token, h.k.shape[0], h.k.shape[1], h.k.shape[2], h.k.shape[3],
                        h.k.shape[4], _DT[h.k.dtype]], dtype=torch.int64, device=dev)
    dist.send(hdr, dst, group=group)
    dist.send(torch.tensor(h.prompt, dtype=torch.int64, device=dev), dst, group=group)
    dist.send(h.k.contiguous(), dst, group=group)
    dist.send(h.v.contiguous(), dst, group=group)


def recv_handoff(src: int, device, group=None) -> KVHandoff:
    hdr = torch.empty(_HDR, dtype=torch.int64, device=device)
    dist.recv(hdr, src, group=group)
    n, first, L, P, Hkv, ps, D, dt = (int(x) for x in hdr.tolist())
    prompt = torch.empty(n, dtype=torch.int64, device=device)
    dist.recv(prompt, src, group=group)
    k = torch.empty(L, P, Hkv, ps, D, dtype=_DT_INV[dt], device=device)
    v = torch.empty_like(k)
    dist.recv(k, src, group=group)
    dist.recv(v, src, group=group)
    return KVHandoff(prompt.tolist(), first, k, v, ps)


class PDCluster:
    """One prefill engine, N decode engines (e.g. one per GPU) in one process."""

    def __init__(self, prefill_engine, decode_engines: list):
        if not decode_engines:
            raise ValueError("no decode engines")
        self.prefill = prefill_engine
        self.decoders = list(decode_engines)
        self.stats = {"handoffs": 0, "handoff_bytes": 0}

    def _pick(self) -> int:
        load = [len(e.running) + len(e.swapped) + len(e.waiting) for e in self.decoders]
        return load.index(min(load))

    def generate(self, prompts: list[list[int]], max_new_tokens: int = 32, sampling: SamplingParams | None = None,
                 stop_ids=()) -> list[list[int]]:
        hs = prefill_handoffs(self.prefill, prompts, sampling)
        reqs = []
        for h in hs:
            e = self.decoders[self._pick()]
            reqs.append((e, adopt(e, h, max_new_tokens, sampling, stop_ids)))
            self.stats["handoffs"] += 1
            self.stats["handoff_bytes"] += h.nbytes
        busy = True
        while busy:
            busy = False
            for e in self.decoders:
                if e.has_work():
                    e.step()
                    busy = True
        return [r.full_output for _, r in reqs]
