"""The serving engine: requests, KV pages, radix prefix reuse, continuous batching.

One ``Engine`` owns one model replica (one GPU, or one tensor-parallel group where every
rank runs the same scheduler deterministically).  ``step()`` is one scheduler iteration:

1. admit waiting requests while KV pages last: look the prompt up in the radix cache
   (whole 16-token pages), take references on the matched pages and allocate pages for
   the rest;
2. prefill the admitted prompt suffixes as one packed ragged chunk (bounded by
   ``max_prefill_tokens``; longer prompts continue in the next iteration);
3. decode one token for every running request in one batched forward (CUDA graph);
4. retire finished requests: their whole pages go into the radix tree for later requests,
   their references are dropped.

Reference behaviour: NativeScheduler (internal/modelengine/nativesched.go:42-227) for the
waiting/running loop, InKernelPlanner.generateReusedContextWithBias
(internal/agent/inkernel_planner.go:1046-1164) for lookup -> clone -> prefill suffix ->
insert -> decode, and KV-block preemption (nativesched_preempt.go) when pages run out.
The reference's device path never reuses prefixes (inkernel_planner.go:1054); this one
always does.
"""
from __future__ import annotations

import dataclasses
import itertools
import math
import time
from typing import Callable

import numpy as np
import torch

from ..config import EngineConfig, ModelConfig
from ..kv import OutOfPages, PagePool, RadixCache
from ..ops import kernels as K
from ..models.runner import KVCache, ModelRunner, PrefillMeta
from ..models.weights import ModelWeights, gguf_source, load_weights, synthetic_source
from .constraints import guided_decode_enabled
from .sampling import SamplingParams, device_sample, needs_counts, pack_params, request_seed, sample


@dataclasses.dataclass
class Request:
    rid: int
    prompt: list[int]
    max_new_tokens: int
    sampling: SamplingParams
    stop_ids: frozenset[int] = frozenset()
    arrival: float = dataclasses.field(default_factory=time.perf_counter)
    # state
    tokens: list[int] = dataclasses.field(default_factory=list)  # prompt + generated
    output: list[int] = dataclasses.field(default_factory=list)
    pages: list[int] = dataclasses.field(default_factory=list)
    n_kv: int = 0            # tokens whose K/V are in ``pages``
    n_cached_hit: int = 0    # prompt tokens served by the radix cache
    first_token_time: float | None = None
    finish_time: float | None = None
    finished: bool = False
    finish_reason: str = ""
    on_token: Callable[[int], None] | None = None
    output_before_preempt: list[int] = dataclasses.field(default_factory=list)  # tokens emitted before a requeue
    swap: tuple | None = None        # (K, V, host bytes) of its pages while swapped out / handed over
    hold_pages: bool = False         # keep the pages at finish (prefill side of a P/D handoff)
    cache_limit: int | None = None   # tokens of this request the radix cache may take (span eviction)
    held_pages: list[int] = dataclasses.field(default_factory=list)
    inflight: int = 0                # decode steps launched for it whose token is not read back yet
    seed: int = 0                    # 64-bit key of its random draws (SamplingParams.seed or derived)

    @property
    def ttft(self) -> float | None:
        return None if self.first_token_time is None else self.first_token_time - self.arrival

    @property
    def full_output(self) -> list[int]:
        """Every token generated so far (across recompute preemptions)."""
        return self.output_before_preempt + self.output


class Engine:
    def __init__(self, weights: ModelWeights, ecfg: EngineConfig | None = None, device: str | torch.device = "cuda",
                 collectives=None, n_pages: int | None = None, max_context: int | None = None, tp_group=None):
        self.ecfg = ecfg or EngineConfig.from_env()
        self.cfg: ModelConfig = weights.cfg
        self.device = torch.device(device)
        self.weights = weights
        ps = self.ecfg.page_size
        if ps != 16:
            raise ValueError("the attention kernels are built for 16-token pages")
        self.max_context = max_context or self.cfg.max_context
        if n_pages is None:
            n_pages = self.ecfg.kv_pages or self._pages_from_memory()
        self.kv = KVCache.allocate(self.cfg.n_layers, n_pages, weights.n_kv_local, self.cfg.head_dim, self.device)
        self.pool = PagePool(n_pages, reserve=1)
        self.radix = RadixCache(self.pool, ps) if self.ecfg.radix_cache else None
        if collectives is None and tp_group is not None and weights.tp_size > 1:
            if self.ecfg.fused_collectives:
                from ..parallel.p2p import P2PTP
                collectives = P2PTP(tp_group, weights, self.ecfg.max_batch, self.device,
                                    spin_limit=self.ecfg.p2p_spin_limit,
                                    max_prefill_tokens=self.ecfg.max_prefill_tokens)
            else:
                from ..parallel.tp import NcclTP
                collectives = NcclTP(tp_group, weights, self.ecfg.max_batch, self.device)
        self.tp_group = tp_group
        offload = None
        if any(L.experts_gate_up is not None and not L.experts_gate_up.buf.is_cuda for L in weights.layers):
            # experts in host memory: their FFNs run on the CPU, which syncs the step with the host at
            # every MoE layer, so no CUDA graphs and no device-resident decode loop
            if weights.tp_size > 1:
                raise NotImplementedError("MoE expert offload runs one GPU per replica (no TP / EP)")
            from ..models.moe_offload import ExpertOffload
            offload = ExpertOffload(weights)
            self.ecfg = dataclasses.replace(self.ecfg, cuda_graph=False, async_decode=False)
        self.runner = ModelRunner(weights, self.kv, max_batch=self.ecfg.max_batch,
                                  max_prefill_tokens=self.ecfg.max_prefill_tokens, max_context=self.max_context,
                                  collectives=collectives, fused_activations=self.ecfg.fused_activations,
                                  attention_merge=self.ecfg.attention_merge, l2_prefetch=self.ecfg.l2_prefetch,
                                  cascade_attention=self.ecfg.cascade_attention, expert_offload=offload)
        self.bt_width = math.ceil(self.max_context / ps)
        if self.ecfg.debug_poison:
            self._poison()
        self.waiting: list[Request] = []
        self.swapped: list[Request] = []   # preempted by swap: resumed (K/V copied back) before new work
        self._swap_bytes = 0
        self.prefilling: list[Request] = []
        self.running: list[Request] = []
        self._rid = itertools.count()
        self.stats = {"prefill_tokens": 0, "prefill_tokens_avoided": 0, "decode_tokens": 0, "steps": 0,
                      "preemptions": 0, "h2d_bytes": 0, "d2h_bytes": 0, "swap_out_pages": 0, "swap_in_pages": 0}
        # weight-load phases (seconds): read, convert (quant-on-load), upload, pack (tile layout), dense
        self.stats.update({"load_" + k + "_s": v for k, v in getattr(weights, "load_profile", {}).items()})
        self._graphs_ready = False
        # device-resident decode loop (_run_decode_async): lanes whose state lives in the runner's
        # static buffers, in row order; the launched step whose tokens are not read back yet
        self._lanes: list[Request] = []
        self._lanes_valid = False
        self._pending: tuple | None = None
        self._n_shared = 0
        self._sampled = False
        self._rb = [torch.zeros(self.ecfg.max_batch + 2, dtype=torch.int32).pin_memory()
                    for _ in range(2)] if self.device.type == "cuda" else []
        self._rb_i = 0

    # ------------------------------------------------------------------------------------
    @staticmethod
    def _tp(tp_group) -> tuple[int, int]:
        if tp_group is None:
            return 0, 1
        import torch.distributed as dist
        return dist.get_rank(tp_group), dist.get_world_size(tp_group)

    @staticmethod
    def _with_lora(source, lora):
        """lora: adapter directories (merged into the weights at load) or a models.lora.LoRASet."""
        if not lora:
            return source
        from ..models.lora import LoRASet, load_peft_adapter, merged_source
        if not isinstance(lora, LoRASet):
            s = LoRASet()
            for d in ([lora] if isinstance(lora, str) else lora):
                load_peft_adapter(d, s)
            lora = s
        return merged_source(source, lora)

    @staticmethod
    def _check_device(cfg: ModelConfig) -> None:
        """Refuse, before any weight is loaded, a model the device kernels cannot run."""
        gap = cfg.device_gap()
        if gap:
            raise NotImplementedError(f"{gap}; run it on the fp32 reference model (serve --cpu)")

    @classmethod
    def from_gguf(cls, path: str, ecfg: EngineConfig | None = None, device="cuda", tp_group=None, lora=None,
                  **kw) -> "Engine":
        r, n = cls._tp(tp_group)
        w = load_weights(cls._with_lora(gguf_source(path), lora), device, tp_rank=r, tp_size=n,
                         prefill_dense=(ecfg or EngineConfig()).prefill_bf16_weights,
                         offload_experts=(ecfg or EngineConfig()).cpu_offload_experts)
        return cls(w, ecfg, device, tp_group=tp_group, **kw)

    @classmethod
    def from_hf(cls, model_dir: str, ecfg: EngineConfig | None = None, device="cuda", tp_group=None, lora=None,
                **kw) -> "Engine":
        """Hugging Face checkpoint directory (safetensors); float matrices are quantized to Q8_0,
        AWQ / GPTQ int4 layers run as G4 blocks."""
        from ..models.hf import hf_source
        r, n = cls._tp(tp_group)
        src = hf_source(model_dir)
        cls._check_device(src[0])
        w = load_weights(cls._with_lora(src, lora), device, tp_rank=r, tp_size=n,
                         prefill_dense=(ecfg or EngineConfig()).prefill_bf16_weights,
                         offload_experts=(ecfg or EngineConfig()).cpu_offload_experts)
        return cls(w, ecfg, device, tp_group=tp_group, **kw)

    @classmethod
    def synthetic(cls, cfg: ModelConfig, mix: str = "q4_k_m", seed: int = 0, ecfg: EngineConfig | None = None,
                  device="cuda", tp_group=None, std: float = 0.02, repeat_layers: bool = False, **kw) -> "Engine":
        """Random-init N(0, std) weights of ``cfg`` quantized on the device (``repeat_layers``: every
        layer shares block 0's weights -- for smoke tests of large architectures)."""
        cls._check_device(cfg)
        r, n = cls._tp(tp_group)
        w = load_weights(synthetic_source(cfg, mix, seed, std=std, device=str(device)), device, tp_rank=r, tp_size=n,
                         prefill_dense=(ecfg or EngineConfig()).prefill_bf16_weights, repeat_layers=repeat_layers,
                         offload_experts=(ecfg or EngineConfig()).cpu_offload_experts)
        return cls(w, ecfg, device, tp_group=tp_group, **kw)

    def shutdown(self) -> None:
        """Release CUDA graphs (they may hold collectives) before the process group goes away."""
        self._drain()
        self.runner._graphs.clear()
        self._graphs_ready = False
        torch.cuda.synchronize(self.device)
        if self.runner.coll is not None and hasattr(self.runner.coll, "close"):
            self.runner.coll.close()

    def _pages_from_memory(self) -> int:
        """KV pages from the free device memory after the weights; fails closed (FitError) when not
        even one sequence of max_context tokens would fit."""
        from ..capacity import FitError, MemoryPlan
        free, _ = torch.cuda.mem_get_info(self.device)
        per = KVCache.bytes_per_page(self.cfg.n_layers, self.weights.n_kv_local, self.cfg.head_dim)
        pages = int(free * self.ecfg.kv_mem_fraction) // per
        need = -(-self.max_context // self.ecfg.page_size) + 1
        if pages < need:
            raise FitError(MemoryPlan(kv=need * per, kv_pages=need), int(free * self.ecfg.kv_mem_fraction))
        return pages

    def warmup_graphs(self, buckets: tuple[int, ...] | None = None) -> None:
        if not self.ecfg.cuda_graph:
            return
        for b in buckets or self.ecfg.graph_batch_buckets:
            if b <= self.ecfg.max_batch:
                self.runner.capture(b, self.bt_width)
                if self.ecfg.spec_k > 0:
                    self.runner.capture(b, self.bt_width, n_layers=self._draft_layers())
        self._graphs_ready = True

    def _draft_layers(self) -> int:
        return max(1, min(self.ecfg.spec_draft_layers, self.cfg.n_layers))

    # ------------------------------------------------------------------------------------
    def add_request(self, prompt: list[int], max_new_tokens: int = 128, sampling: SamplingParams | None = None,
                    stop_ids=(), on_token=None) -> Request:
        if not prompt:
            raise ValueError("empty prompt")
        if len(prompt) + max_new_tokens > self.max_context:
            raise ValueError(f"prompt {len(prompt)} + {max_new_tokens} new tokens exceeds context {self.max_context}")
        r = Request(next(self._rid), list(prompt), max_new_tokens, sampling or SamplingParams(),
                    frozenset(stop_ids), on_token=on_token)
        r.seed = (int(r.sampling.seed) & 0xFFFFFFFFFFFFFFFF if r.sampling.seed is not None
                  else request_seed(self.ecfg.seed, r.rid))
        r.tokens = list(prompt)
        self.waiting.append(r)
        return r

    def has_work(self) -> bool:
        return bool(self.waiting or self.prefilling or self.running or self.swapped or self._pending)

    def _alloc(self, n: int) -> list[int]:
        if n <= 0:
            return []
        if self.pool.n_free() < n and self.radix is not None:
            self.radix.evict(n - self.pool.n_free())
        return self.pool.alloc(n)

    def _resume_swapped(self) -> bool:
        """Swap preempted requests back in (oldest first); False while one does not fit yet."""
        while self.swapped and len(self.running) + len(self.prefilling) < self.ecfg.max_batch:
            r = self.swapped[0]
            k, v, host_bytes = r.swap
            try:
                pages = self._alloc(k.shape[1])
            except OutOfPages:
                return False
            self.swapped.pop(0)
            idx = torch.tensor(pages, dtype=torch.long).to(self.device, non_blocking=True)
            self.kv.k.index_copy_(1, idx, k.to(self.device, non_blocking=True))
            self.kv.v.index_copy_(1, idx, v.to(self.device, non_blocking=True))
            self.stats["swap_in_pages"] += len(pages)
            self.stats["h2d_bytes"] += 2 * k.numel() * k.element_size()
            self._swap_bytes -= host_bytes
            r.swap = None
            r.pages = pages
            self.running.append(r)
        return not self.swapped

    def _admit(self) -> None:
        ps = self.ecfg.page_size
        if not self._resume_swapped():
            return   # swapped requests go first: admitting new work would only evict them again
        while self.waiting and len(self.running) + len(self.prefilling) < self.ecfg.max_batch:
            r = self.waiting[0]
            hit, pages = 0, []
            if self.radix is not None:
                # keep at least one prompt token to prefill: its logits give the first output token
                hit, pages = self.radix.lookup(r.prompt, max_tokens=len(r.prompt) - 1)
            need = math.ceil(len(r.prompt) / ps) - len(pages)
            try:
                new = self._alloc(need)
            except OutOfPages:
                self.pool.release(pages)
                if not self.running and not self.prefilling:
                    raise
                break
            self.waiting.pop(0)
            r.pages = pages + new
            r.n_kv = hit
            r.n_cached_hit = hit
            self.stats["prefill_tokens_avoided"] += hit
            self.prefilling.append(r)

    # ------------------------------------------------------------------------------------
    def _run_prefill(self) -> None:
        budget = self.ecfg.max_prefill_tokens
        chunk: list[tuple[Request, int, int]] = []
        for r in self.prefilling:
            if budget <= 0:
                break
            n = min(len(r.prompt) - r.n_kv, budget)
            chunk.append((r, r.n_kv, n))
            budget -= n
        if not chunk:
            return
        ps = self.ecfg.page_size
        ids, pos, slot, qlens, pos0s, last = [], [], [], [], [], []
        W = max(len(r.pages) for r, s, n in chunk)
        bt = np.zeros((len(chunk), max(W, 1)), dtype=np.int32)
        t = 0
        for k, (r, s, n) in enumerate(chunk):
            ids.extend(r.prompt[s:s + n])
            p = np.arange(s, s + n)
            pos.extend(p.tolist())
            pg = np.asarray(r.pages, dtype=np.int64)
            slot.extend((pg[p // ps] * ps + p % ps).tolist())
            bt[k, :len(r.pages)] = r.pages
            qlens.append(n)
            pos0s.append(s)
            t += n
            last.append(t - 1)
        dev = self.device
        to = lambda a: torch.tensor(a, dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
        meta = PrefillMeta.build(qlens, pos0s, dev)
        self.stats["h2d_bytes"] += 4 * (3 * len(ids) + len(last) + bt.size + 3 * len(qlens) + 2 * meta.n_tiles)
        logits = self.runner.prefill(to(ids), to(pos), to(slot), torch.from_numpy(bt).pin_memory().to(dev, non_blocking=True),
                                     meta, to(last))
        self.stats["prefill_tokens"] += t
        done = []
        for k, (r, s, n) in enumerate(chunk):
            r.n_kv = s + n
            if r.n_kv == len(r.prompt):
                done.append((k, r))
        if done:
            rows = torch.tensor([k for k, _ in done], device=dev)
            toks = self._sample_rows(logits.index_select(0, rows), [r for _, r in done])
            self.stats["d2h_bytes"] += 8 * len(done)
            now = time.perf_counter()
            for (k, r), tok in zip(done, toks):
                self.prefilling.remove(r)
                r.first_token_time = now
                self._emit(r, tok)
                if not r.finished:
                    self.running.append(r)

    def _emit(self, r: Request, tok: int) -> None:
        r.output.append(tok)
        r.tokens.append(tok)
        if r.on_token is not None:
            r.on_token(tok)
        if tok in r.stop_ids:
            self._finish(r, "stop")
        elif len(r.output) >= r.max_new_tokens:
            self._finish(r, "length")

    def _finish(self, r: Request, reason: str) -> None:
        r.finished = True
        r.finish_reason = reason
        r.finish_time = time.perf_counter()
        if self.radix is not None:
            # the K/V of tokens[:n_kv] is in the pages; the last sampled token was never fed
            self.radix.insert(r.tokens[:self._cacheable(r)], r.pages)
        if r.hold_pages:
            r.held_pages = r.pages   # the caller exports their K/V, then releases them
        else:
            self.pool.release(r.pages)
        r.pages = []

    def _poison(self) -> None:
        """Debug: NaN in every float scratch buffer and a large finite sentinel in the KV cache, so a
        kernel that reads scratch it did not write, or K/V positions its mask should exclude, changes
        the outputs (masked positions are multiplied by an exact zero, which a finite sentinel keeps)."""
        nan = float("nan")
        rn = self.runner
        for t in (rn.attn_ws, rn.qkv, rn.q, rn.h, rn.tmp, rn.logits, rn.x):
            t.fill_(nan)
        part, _ = K.tgemv_workspace(self.device)
        part.fill_(nan)
        self.kv.k.fill_(3.0e4)
        self.kv.v.fill_(3.0e4)

    @staticmethod
    def _masked(r: Request) -> bool:
        """Guided decoding: its token mask is computed on the host, so it samples on the host."""
        return r.sampling.mask is not None and guided_decode_enabled()

    def _sample_rows(self, logits: torch.Tensor, reqs: list[Request]) -> list[int]:
        """One token per logit row (modified in place): the device sampler, or the host path when a
        request's guided-decoding mask is active."""
        if any(self._masked(r) for r in reqs):
            return sample(self._capped(logits), [r.sampling for r in reqs], reqs)
        if all(r.sampling.greedy for r in reqs):
            return torch.argmax(logits, dim=-1).tolist()
        return device_sample(logits, self.cfg.vocab_size, [r.sampling for r in reqs],
                             [len(r.full_output) for r in reqs], [r.seed for r in reqs],
                             [r.full_output for r in reqs], self.cfg.final_softcap)

    def _capped(self, logits: torch.Tensor) -> torch.Tensor:
        """Final-logit soft-capping (Gemma-2) before sampling; greedy argmax is unaffected by it."""
        c = self.cfg.final_softcap
        return c * torch.tanh(logits / c) if c > 0 else logits

    @staticmethod
    def _cacheable(r: Request) -> int:
        return r.n_kv if r.cache_limit is None else min(r.n_kv, r.cache_limit)

    def evict_span(self, r: Request, start: int, end: int) -> int:
        """Remove token positions [start, end) from a request's K/V between steps: later positions
        move down by end - start with their keys re-rotated to the new positions, so the model can no
        longer attend to the span.  Pages from the span's first page on are rewritten into fresh
        pages (shared prefix pages are never modified).  Returns the number of positions removed.

        The K/V of tokens after the span were computed while the span was visible, so from then on
        only the tokens before the span may enter the radix cache."""
        from ..models.rope import inv_freq
        from ..ops import kernels as K
        self._drain()
        self._lanes_valid = False   # pages and positions change under the resident lanes
        if r.finished or r.swap is not None or r in self.waiting or r in self.prefilling:
            raise ValueError("evict_span: the request must be decoding (between steps)")
        if not 0 <= start < end <= r.n_kv:
            raise ValueError(f"evict_span: span [{start}, {end}) outside the cached {r.n_kv} positions")
        ps, n, N = self.ecfg.page_size, end - start, r.n_kv
        first = start // ps
        new_len = N - n
        fresh = self._alloc(-(-new_len // ps) - first) if new_len > first * ps else []
        q = np.arange(first * ps, new_len)
        src = np.where(q < start, q, q + n)
        old = np.asarray(r.pages, dtype=np.int64)
        dst_pages = np.asarray(fresh, dtype=np.int64)
        src_slot = old[src // ps] * ps + src % ps
        dst_slot = dst_pages[q // ps - first] * ps + q % ps if len(q) else np.zeros(0, np.int64)
        inv, _ = inv_freq(self.cfg.head_dim, self.cfg.rope_theta, self.cfg.rope_scaling, self.cfg.max_context)
        ang = inv * float(n)
        dev = self.device
        K.kv_move(self.kv, torch.from_numpy(src_slot.astype(np.int32)).to(dev),
                  torch.from_numpy(dst_slot.astype(np.int32)).to(dev),
                  torch.from_numpy((q >= start).astype(np.uint8)).to(dev),
                  torch.cos(ang).float().to(dev), torch.sin(ang).float().to(dev))
        self.pool.release(r.pages[first:])
        r.pages = r.pages[:first] + fresh
        survivors_after = N - end
        r.tokens = r.tokens[:start] + r.tokens[end:]
        r.n_kv = new_len
        limit = start if survivors_after > 0 else new_len
        r.cache_limit = limit if r.cache_limit is None else min(r.cache_limit, limit)
        self.stats["evicted_positions"] = self.stats.get("evicted_positions", 0) + n
        return n

    def _ensure_pages(self, r: Request, last_pos: int) -> bool:
        need = last_pos // self.ecfg.page_size + 1 - len(r.pages)
        if need > 0:
            try:
                r.pages.extend(self._alloc(need))
            except OutOfPages:
                self._preempt(r)
                return False
        return True

    def _async_ok(self) -> bool:
        return (self.ecfg.async_decode and self._graphs_ready and self.ecfg.spec_k == 0
                and not any(self._masked(r) for r in self.running))

    def _run_decode(self) -> None:
        if self.running and self._async_ok():
            if self._run_decode_async():
                return
        self._drain()
        self._lanes_valid = False    # the synchronous step rewrites the static inputs
        self._run_decode_sync()

    # ---- device-resident decode loop -------------------------------------------------------
    def _need(self, r: Request) -> int:
        """Decode steps still to launch for r (its remaining tokens minus those in flight)."""
        return 0 if r.finished else r.max_new_tokens - len(r.output) - r.inflight

    def _run_decode_async(self) -> bool:
        """One decode step of the device-resident loop; False when it cannot run (out of pages).

        The lanes' inputs stay on the device between steps (the graph's last kernel advances them);
        this launches step t, then reads back step t - 1's tokens, so the host's bookkeeping overlaps
        the GPU's work.  The lane set is re-uploaded only when it changes (a request joined or
        finished), after the in-flight step was read back.  A lane that stops on a stop token runs
        one extra step whose token is dropped; stops by length are known ahead and cost nothing."""
        ps, W = self.ecfg.page_size, self.bt_width
        lanes = [r for r in self.running if self._need(r) > 0]
        if [id(r) for r in lanes] != [id(r) for r in self._lanes] or not self._lanes_valid:
            self._drain()
            lanes = [r for r in self.running if self._need(r) > 0]
            if not lanes:
                return True
            if not self._map_pages(lanes, None):
                return False
            self._upload_lanes(lanes)
        else:
            patches: list[int] = []
            if not self._map_pages(lanes, patches):
                return False
            if patches:
                _, bt = self.runner.lane_state(W)
                iv = torch.tensor(patches, dtype=torch.int32).pin_memory().to(self.device, non_blocking=True)
                K.scatter_i32(bt, iv, len(patches) // 2)
                self.stats["h2d_bytes"] += 4 * len(patches)
        B = len(lanes)
        self.runner.replay_resident(B, self._n_shared, self._sampled)
        buf = self._rb[self._rb_i]
        self._rb_i ^= 1
        rn = self.runner
        buf[:B].copy_(rn.status[:B], non_blocking=True)
        buf[-2:].copy_(rn.status[rn.max_batch:rn.max_batch + 2], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        for r in lanes:
            r.n_kv += 1
            r.inflight += 1
        prev, self._pending = self._pending, (ev, buf, list(lanes))
        self.stats["decode_tokens"] += B
        self.stats["d2h_bytes"] += 4 * (B + 2)
        if prev is not None:
            self._collect(prev)
        return True

    def _map_pages(self, lanes: list[Request], patches: list[int] | None) -> bool:
        """Pages for the position each lane feeds now and, when it runs again, the next one (the
        graph computes that slot on the device).  ``patches`` collects (flat index, page) pairs of
        new block-table entries of resident lanes.  False (nothing changed for the lane that failed)
        when the pool runs dry: the caller falls back to the synchronous step, which preempts."""
        ps, W = self.ecfg.page_size, self.bt_width
        for b, r in enumerate(lanes):
            last = r.n_kv + (1 if self._need(r) > 1 else 0)
            need = min(last, self.max_context - 1) // ps + 1 - len(r.pages)
            if need > 0:
                try:
                    new = self._alloc(need)
                except OutOfPages:
                    return False
                if patches is not None:
                    for j, pg in enumerate(new):
                        patches += [b * W + len(r.pages) + j, pg]
                r.pages.extend(new)
        return True

    def _upload_lanes(self, lanes: list[Request]) -> None:
        """Write every lane's state (and idle rows after them) into the runner's static inputs."""
        ps, W, mb = self.ecfg.page_size, self.bt_width, self.ecfg.max_batch
        vec = np.zeros((4, mb), np.int32)
        vec[2, :] = -1
        vec[3, :] = 1
        bt = np.zeros((mb, W), np.int32)
        for b, r in enumerate(lanes):
            p = r.n_kv
            vec[0, b] = r.tokens[-1]
            vec[1, b] = p
            vec[2, b] = r.pages[p // ps] * ps + p % ps
            vec[3, b] = p + 1
            bt[b, :len(r.pages)] = r.pages
        dv, dbt = self.runner.lane_state(W)
        dv.copy_(torch.from_numpy(vec).pin_memory(), non_blocking=True)
        dbt.copy_(torch.from_numpy(bt).pin_memory(), non_blocking=True)
        self.stats["h2d_bytes"] += vec.nbytes + bt.nbytes
        # sampled lanes: the device sampler's rows (parameters, bias lists, generated-token counts)
        B = len(lanes)
        rn = self.runner
        self._sampled = any(not r.sampling.greedy for r in lanes)
        if self._sampled:
            P, tok, val = pack_params([r.sampling for r in lanes], [len(r.full_output) for r in lanes],
                                      [r.seed for r in lanes])
            rn.samp_params[:B].copy_(torch.from_numpy(P).pin_memory(), non_blocking=True)
            if len(tok):
                rn.bias_tok[:len(tok)].copy_(torch.from_numpy(tok).pin_memory(), non_blocking=True)
                rn.bias_val[:len(val)].copy_(torch.from_numpy(val).pin_memory(), non_blocking=True)
            if needs_counts([r.sampling for r in lanes]):
                from .sampling import count_rows
                rn.counts[:B].copy_(count_rows([r.full_output for r in lanes], self.cfg.vocab_size, self.device))
            self.stats["h2d_bytes"] += P.nbytes + tok.nbytes + val.nbytes
        # the lanes' common leading pages (a radix-shared prefix) cannot change while the lane set is
        # fixed: new pages are private to their lane, and every lane's context only grows
        self._n_shared = self._shared_pages(bt[:B], vec[3, :B]) if self.runner.cascade_ok(B) else 0
        if self._n_shared >= self.runner.min_shared_pages:
            self.runner.shared_pages.copy_(torch.tensor([self._n_shared], dtype=torch.int32).pin_memory(),
                                           non_blocking=True)
        self._lanes = list(lanes)
        self._lanes_valid = True

    def _collect(self, pending) -> None:
        """Read back one launched step: emit each lane's token (dropped for a lane that stopped
        meanwhile), fail loudly on a device error word."""
        ev, buf, lanes = pending
        ev.synchronize()
        vals = buf.tolist()
        kerr, cerr = vals[-2], vals[-1]
        for r in lanes:
            r.inflight -= 1
        if kerr or cerr:
            self._device_error(kerr, cerr)
        for b, r in enumerate(lanes):
            if not r.finished:
                self._emit(r, int(vals[b]))
        self.running = [r for r in self.running if not r.finished]

    def _drain(self) -> None:
        if self._pending is not None:
            p, self._pending = self._pending, None
            self._collect(p)

    def _device_error(self, kerr: int, cerr: int) -> None:
        """A kernel's bounded wait expired (or it saw an out-of-range id): the step's outputs are not
        trustworthy.  Every running request fails and the engine refuses further steps."""
        from ..parallel.errors import DeviceStepError
        msg = (f"decode step failed on the device: kernel error word {kerr}, collective error word {cerr} "
               "(kernel: 1 = a bounded wait expired, 2 = an index out of range, 4 = a peer rank never arrived at a "
               "fused all-reduce; collective: 1 = a peer rank never arrived at a barrier)")
        for r in list(self.running):
            r.finished = True
            r.finish_reason = "error"
        self.running = []
        raise DeviceStepError(msg, kerr, cerr)

    def _run_decode_sync(self) -> None:
        if not self.running:
            return
        ps = self.ecfg.page_size
        k = self.ecfg.spec_k
        if k > 0 and all(r.sampling.greedy for r in self.running):
            lanes = [r for r in list(self.running)
                     if self._ensure_pages(r, min(r.n_kv + k, self.max_context - 1))]
            if lanes:
                self._run_decode_spec(lanes, k)
            return
        lanes = []
        for r in list(self.running):
            p = r.n_kv  # position of the token being fed (the last sampled one)
            if p // ps >= len(r.pages):
                try:
                    r.pages.extend(self._alloc(1))
                except OutOfPages:
                    self._preempt(r)
                    continue
            lanes.append(r)
        if not lanes:
            return
        B = len(lanes)
        W = self.bt_width
        ids = np.empty(B, np.int32)
        pos = np.empty(B, np.int32)
        slot = np.empty(B, np.int32)
        ctx = np.empty(B, np.int32)
        bt = np.zeros((B, W), np.int32)
        for k, r in enumerate(lanes):
            p = r.n_kv
            ids[k] = r.tokens[-1]
            pos[k] = p
            slot[k] = r.pages[p // ps] * ps + p % ps
            ctx[k] = p + 1
            bt[k, :len(r.pages)] = r.pages
        dev = self.device
        shared = np.array([self._shared_pages(bt, ctx)], np.int32)
        h = torch.from_numpy(np.concatenate([ids, pos, slot, ctx, shared])).pin_memory()
        d = h.to(dev, non_blocking=True)
        btd = torch.from_numpy(bt).pin_memory().to(dev, non_blocking=True)
        greedy = all(r.sampling.greedy for r in lanes)
        if not greedy and self.runner.coll is not None:
            # the tensor-parallel greedy graph never gathers the full logits: run the step eagerly
            self.runner.decode_eager(d[0:B], d[B:2 * B], d[2 * B:3 * B], btd, d[3 * B:4 * B], B, greedy=False)
            out = self.runner.next_ids[:B]
        else:
            out = self.runner.decode(d[0:B], d[B:2 * B], d[2 * B:3 * B], btd, d[3 * B:4 * B], B,
                                     use_graph=self._graphs_ready, shared=d[4 * B:4 * B + 1],
                                     n_shared=int(shared[0]))
        self.stats["h2d_bytes"] += h.numel() * 4 + bt.size * 4
        mb = self.runner.max_batch
        kerr, cerr = self.runner.status[mb:mb + 2].tolist()
        if kerr or cerr:
            self._device_error(kerr, cerr)
        if greedy:
            toks = out.cpu().tolist()
            self.stats["d2h_bytes"] += 4 * B + 8
        else:
            toks = self._sample_rows(self.runner.logits[:B], lanes)
            self.stats["d2h_bytes"] += 8 * B
        self.stats["decode_tokens"] += B
        for r, tok in zip(lanes, toks):
            r.n_kv += 1
            self._emit(r, tok)
        self.running = [r for r in self.running if not r.finished]

    def _shared_pages(self, bt: np.ndarray, ctx: np.ndarray) -> int:
        """Leading block-table pages that are the same physical page in every lane and lie before
        every lane's current page (the radix-shared prefix of the batch): cascade attention reads
        them once for all lanes."""
        B = bt.shape[0]
        if B < 2:
            return 0
        k = int((ctx.min() - 1) // self.ecfg.page_size)
        if k <= 0:
            return 0
        same = (bt[:, :k] == bt[0:1, :k]).all(axis=0)
        return int(k if same.all() else np.argmin(same))

    def _run_decode_spec(self, lanes: list[Request], k: int) -> None:
        """Greedy speculative decode (reference: spec.SpeculativeGreedy, internal/spec/spec.go:214-300).

        Drafts come from ``spec_drafter``: "self" (the target's first layers + LM head, sharing its KV
        pages), "lookup" (n-gram prompt lookup over the request's own context, no model), "multi"
        (per request, whichever of the two has been accepted more) or "tree" (several lookup
        continuations verified as a tree, ``_run_decode_tree``).  The target verifies all k+1
        positions of a chain in one forward, each position running as its own attention lane with a
        causal context length; the longest agreeing prefix plus the target's next token are kept,
        and the KV of rejected positions is dropped by truncating the lane's KV length (its pages are
        simply overwritten later).  The output is identical to plain greedy decoding."""
        mode = self.ecfg.spec_drafter
        if mode == "tree":
            self._run_decode_tree(lanes, k)
            return
        ps, dev, B, W = self.ecfg.page_size, self.device, len(lanes), self.bt_width
        bt = np.zeros((B, W), np.int32)
        p0 = np.array([r.n_kv for r in lanes], np.int64)
        for b, r in enumerate(lanes):
            bt[b, :len(r.pages)] = r.pages
        pages = [np.asarray(r.pages, np.int64) for r in lanes]

        def slots(pos):
            return np.array([pages[b][pos[b] // ps] * ps + pos[b] % ps for b in range(B)], np.int32)

        btd = torch.from_numpy(bt).pin_memory().to(dev, non_blocking=True)
        cur = [r.tokens[-1] for r in lanes]
        self_drafts = None
        if mode in ("self", "multi"):
            feed = [torch.tensor(cur, dtype=torch.int32).to(dev)]
            Ld = self._draft_layers()
            for j in range(k):
                pos = np.minimum(p0 + j, self.max_context - 1)
                h = torch.from_numpy(np.concatenate([pos.astype(np.int32), slots(pos), (pos + 1).astype(np.int32)]))
                d = h.pin_memory().to(dev, non_blocking=True)
                out = self.runner.decode(feed[-1], d[0:B], d[B:2 * B], btd, d[2 * B:3 * B], B,
                                         use_graph=self._graphs_ready, n_layers=Ld)
                feed.append(out.clone())
            self_drafts = torch.stack(feed[1:], 1).cpu().numpy()
        drafts = np.zeros((B, k), np.int64)
        for b, r in enumerate(lanes):
            if mode == "self":
                drafts[b] = self_drafts[b]
                continue
            dr = self._drafter(r)
            if mode == "multi":
                dr.members[1][1].pending = list(self_drafts[b])
            prop = list(dr.draft(k))[:k]
            drafts[b] = prop + [cur[b]] * (k - len(prop))    # pad: a rejected filler, never a loss
        toks_h = np.concatenate([np.asarray(cur, np.int64)[:, None], drafts], 1).astype(np.int32)
        toks = torch.from_numpy(toks_h.reshape(-1)).pin_memory().to(dev, non_blocking=True)
        V = B * (k + 1)
        vpos = (p0[:, None] + np.arange(k + 1)[None, :]).reshape(-1)
        vpos = np.minimum(vpos, self.max_context - 1)
        vslot = np.array([pages[i // (k + 1)][vpos[i] // ps] * ps + vpos[i] % ps for i in range(V)], np.int32)
        h = torch.from_numpy(np.concatenate([vpos.astype(np.int32), vslot, (vpos + 1).astype(np.int32)]))
        d = h.pin_memory().to(dev, non_blocking=True)
        vbt = btd.repeat_interleave(k + 1, dim=0)
        tgt = self.runner.decode(toks, d[0:V], d[V:2 * V], vbt, d[2 * V:3 * V], V, use_graph=self._graphs_ready)
        t_host = tgt.view(B, k + 1).cpu().numpy()
        self.stats["spec_steps"] = self.stats.get("spec_steps", 0) + 1
        self.stats["h2d_bytes"] += bt.size * 4 + (k + 1) * 12 * B + 12 * V
        self.stats["d2h_bytes"] += 8 * V
        for b, r in enumerate(lanes):
            acc = 0
            while acc < k and drafts[b, acc] == t_host[b, acc]:
                acc += 1
            self.stats["spec_proposed"] = self.stats.get("spec_proposed", 0) + k
            self.stats["spec_accepted"] = self.stats.get("spec_accepted", 0) + acc
            emitted = [int(x) for x in drafts[b, :acc]] + [int(t_host[b, acc])]
            if mode != "self":
                self._drafter(r).commit(emitted)
            for t in emitted:
                if r.finished:
                    break
                r.n_kv += 1
                self._emit(r, t)
        self.stats["decode_tokens"] += B
        self.running = [r for r in self.running if not r.finished]

    def _drafter(self, r: Request):
        """The request's drafter, created on first use over its tokens so far (kept in step with
        the committed tokens by the spec paths)."""
        from .drafters import LookupDrafter, MultiDrafter, TreeLookupDrafter
        dr = getattr(r, "drafter", None)
        if dr is None:
            mode = self.ecfg.spec_drafter
            if mode == "tree":
                dr = TreeLookupDrafter(r.tokens, width=self.ecfg.spec_tree_width)
            elif mode == "multi":
                dr = MultiDrafter([("lookup", LookupDrafter(r.tokens)), ("self", _Pending())])
            else:
                dr = LookupDrafter(r.tokens)
            r.drafter = dr
        return dr

    def _run_decode_tree(self, lanes: list[Request], depth: int) -> None:
        """Greedy tree speculation (reference: spec.VerifyTree, internal/spec/verify.go:54-122).

        Each lane's drafter proposes a token tree; every root-to-leaf path becomes a chain of
        decode lanes (its positions base .. base + d, each lane attending causally along its own
        path).  A chain gets private copies of the request's partial tail page, so sibling
        branches writing the same positions never collide.  The accepted path is the longest one
        whose tokens equal the target's greedy tokens; the pages of a chain holding it replace
        the request's tail pages (no copy of the accepted K/V), the rest are released."""
        from ..ops import kernels as K
        from .drafters import accept_tree
        ps, dev, W = self.ecfg.page_size, self.device, self.bt_width
        lane_tok, lane_pos, lane_slot, lane_bt = [], [], [], []
        plans = []
        budget = self.ecfg.max_batch
        src_slots, dst_slots = [], []
        for r in lanes:
            dr = self._drafter(r)
            tree = dr.propose(depth)
            base = r.n_kv
            pg0 = base // ps
            leaves = tree.leaves() if tree.tokens else []
            chains = [tree.path(l) for l in leaves] or [[]]
            chains = [c[:max(0, min(len(c), self.max_context - 1 - base))] for c in chains]
            # at most the lanes that still fit this step (a chain of d nodes takes d + 1 lanes)
            keep = []
            for c in chains:
                if budget - (len(c) + 1) < 0:
                    break
                keep.append(c)
                budget -= len(c) + 1
            if not keep:
                keep = [[]]
            priv = []
            for c in keep:
                n_tail = (base + len(c)) // ps - pg0 + 1
                try:
                    pages = self._alloc(n_tail)
                except OutOfPages:
                    for p_ in priv:
                        self.pool.release(p_)
                    self._release_plans(plans)
                    self._run_decode_sync_plain(lanes)
                    return
                priv.append(pages)
                for q in range(pg0 * ps, base):          # the committed rows of the partial tail page
                    src_slots.append(r.pages[q // ps] * ps + q % ps)
                    dst_slots.append(pages[0] * ps + q % ps)
            plans.append((r, tree, base, pg0, keep, priv, len(lane_tok)))
            for c, pages in zip(keep, priv):
                row = np.zeros(W, np.int32)
                row[:pg0] = r.pages[:pg0]
                row[pg0:pg0 + len(pages)] = pages
                feed = [r.tokens[-1]] + [tree.tokens[i] for i in c]
                for j, t in enumerate(feed):
                    p = base + j
                    lane_tok.append(t)
                    lane_pos.append(p)
                    lane_slot.append(pages[p // ps - pg0] * ps + p % ps)
                    lane_bt.append(row)
        if src_slots:
            z = torch.zeros(len(src_slots), dtype=torch.uint8, device=dev)
            one = torch.ones(self.cfg.head_dim // 2, dtype=torch.float32, device=dev)
            K.kv_move(self.kv, torch.tensor(src_slots, dtype=torch.int32, device=dev),
                      torch.tensor(dst_slots, dtype=torch.int32, device=dev), z, one, one * 0)
        V = len(lane_tok)
        to = lambda a: torch.from_numpy(np.asarray(a, np.int32)).pin_memory().to(dev, non_blocking=True)
        tgt = self.runner.decode(to(lane_tok), to(lane_pos), to(lane_slot), to(np.stack(lane_bt)),
                                 to(np.asarray(lane_pos) + 1), V, use_graph=self._graphs_ready)
        t_host = tgt.cpu().numpy()
        self.stats["spec_steps"] = self.stats.get("spec_steps", 0) + 1
        self.stats["h2d_bytes"] += 16 * V + V * W * 4
        self.stats["d2h_bytes"] += 4 * V
        for r, tree, base, pg0, keep, priv, off in plans:
            node_tgt = [0] * len(tree.tokens)
            root_tgt = int(t_host[off])
            o = off
            for c in keep:
                for j, i in enumerate(c):
                    node_tgt[i] = int(t_host[o + 1 + j])
                o += len(c) + 1
            path, committed = accept_tree(tree, root_tgt, node_tgt)
            win = next(ci for ci, c in enumerate(keep) if c[:len(path)] == path)
            self.stats["spec_proposed"] = self.stats.get("spec_proposed", 0) + len(tree.tokens)
            self.stats["spec_accepted"] = self.stats.get("spec_accepted", 0) + len(path)
            # the winning chain's pages hold the committed rows and the accepted path's K/V
            self.pool.release(r.pages[pg0:])
            r.pages = r.pages[:pg0] + priv[win]
            for ci, pages in enumerate(priv):
                if ci != win:
                    self.pool.release(pages)
            r.drafter.commit(committed)
            for t in committed:
                if r.finished:
                    break
                r.n_kv += 1
                self._emit(r, int(t))
        self.stats["decode_tokens"] += len(lanes)
        self.running = [r for r in self.running if not r.finished]

    def _release_plans(self, plans) -> None:
        for _, _, _, _, _, priv, _ in plans:
            for pages in priv:
                self.pool.release(pages)

    def _run_decode_sync_plain(self, lanes: list[Request]) -> None:
        """Fallback of the tree path when private pages run out: one plain decode step."""
        k, self.ecfg.spec_k = self.ecfg.spec_k, 0
        try:
            self._run_decode_sync()
        finally:
            self.ecfg.spec_k = k

    def _preempt(self, r: Request) -> None:
        """Out of pages: give this request's pages back.  Swap mode copies their K/V to pinned host
        memory and resumes the request later with the K/V copied back (no recompute); otherwise
        (or when the swap space is full) the request is recomputed later, its finished prefix in
        the radix cache so the recompute is cheap."""
        self.stats["preemptions"] += 1
        self.running.remove(r)
        nbytes = 2 * len(r.pages) * self.kv.k[:, :1].numel() * self.kv.k.element_size()
        if (self.ecfg.preempt_mode == "swap" and r.pages
                and self._swap_bytes + nbytes <= self.ecfg.swap_space_gb * (1 << 30)):
            idx = torch.tensor(r.pages, dtype=torch.long).to(self.device, non_blocking=True)
            host = []
            for t in (self.kv.k, self.kv.v):
                g = t.index_select(1, idx)   # [L, n, Hkv, page, D] gathered on the device
                h = torch.empty(g.shape, dtype=g.dtype, pin_memory=True)
                h.copy_(g, non_blocking=True)   # stream-ordered before the pages are reused
                host.append(h)
            r.swap = (host[0], host[1], nbytes)
            self._swap_bytes += nbytes
            self.stats["swap_out_pages"] += len(r.pages)
            self.stats["d2h_bytes"] += nbytes
            self.pool.release(r.pages)
            r.pages = []
            self.swapped.append(r)
            return
        if self.radix is not None:
            self.radix.insert(r.tokens[:self._cacheable(r)], r.pages)
        self.pool.release(r.pages)
        r.pages = []
        r.cache_limit = None   # recomputed from its tokens: its K/V will be plain again
        r.prompt = list(r.tokens)
        r.max_new_tokens -= len(r.output)
        r.output_before_preempt = r.output_before_preempt + r.output
        r.output = []
        r.n_kv = 0
        self.waiting.insert(0, r)

    def step(self) -> None:
        self._admit()
        self._run_prefill()
        self._run_decode()
        self.stats["steps"] += 1

    def run_until_done(self, reqs: list[Request] | None = None) -> None:
        while self.has_work():
            self.step()
            if reqs is not None and all(r.finished for r in reqs):
                break

    def generate(self, prompts: list[list[int]], max_new_tokens: int = 32, sampling: SamplingParams | None = None,
                 stop_ids=()) -> list[list[int]]:
        reqs = [self.add_request(p, max_new_tokens, sampling, stop_ids) for p in prompts]
        self.run_until_done(reqs)
        return [r.full_output for r in reqs]


class _Pending:
    """A multi-drafter member whose proposal for the round (the batch's self-draft) is set before
    the round's draft call."""

    def __init__(self):
        self.pending: list[int] = []

    def draft(self, k: int) -> list[int]:
        return [int(t) for t in self.pending[:k]]

    def commit(self, tokens: list[int]) -> None:
        pass
