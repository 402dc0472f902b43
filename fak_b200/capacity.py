"""Capacity / memory planning: what a model, its KV cache and its workspaces take on each GPU.

A ``MemoryPlan`` adds up, per rank, the device bytes of a serving configuration:

* quantized weights (GGML blocks at the device row pitch) and their tile-packed decode copy;
* the bf16 copies the prefill GEMMs read (``EngineConfig.prefill_bf16_weights``);
* the paged KV cache (bf16 K and V, 16-token pages) for the requested context x batch;
* decode / prefill activation workspaces and the split-K / attention scratch.

``check_fits`` refuses a plan that does not fit the device budget with a typed ``FitError``
naming the largest items, before anything is allocated; ``max_context`` sizes the context (or
the KV pages) that a budget leaves.  Expert parallelism divides the expert weights over the
ranks, tensor parallelism the attention heads, FFN rows and vocabulary.

Reference: internal/compute/capacity.go (MemoryPlan / MemoryDemand :60-365, FitsOnDevice and
RefuseMemoryPlanIfTooBig :523-706, DeviceAllocError :776, the EP per-rank plan :206-266) and
AutoSizeContextPlan (internal/compute/contextsizer.go).
"""
from __future__ import annotations

import dataclasses
import math

from .config import ModelConfig

# bytes per weight of the device block formats (GGML blocks; Q4_K_M mixes mostly Q4_K with some Q6_K)
BYTES_PER_WEIGHT = {"q4_k": 144 / 256, "q6_k": 210 / 256, "q8_0": 34 / 32, "f16": 2.0, "bf16": 2.0, "f32": 4.0}
MIX_WEIGHT_BYTES = {"q4_k_m": 0.60, "q8_0": 34 / 32, "q6_k": 210 / 256, "f16": 2.0, "bf16": 2.0}
PAGE_TOKENS = 16


class FitError(RuntimeError):
    """A serving plan does not fit the device memory budget (nothing was allocated)."""

    def __init__(self, plan: "MemoryPlan", budget: int):
        self.plan, self.budget = plan, budget
        top = sorted(plan.items().items(), key=lambda kv: -kv[1])[:3]
        items = ", ".join(f"{k} {v / 2**30:.2f} GiB" for k, v in top)
        super().__init__(f"plan needs {plan.total / 2**30:.2f} GiB per GPU, budget {budget / 2**30:.2f} GiB "
                         f"(largest: {items})")


@dataclasses.dataclass
class MemoryPlan:
    weights: int = 0          # quantized blocks
    tile_packed: int = 0      # decode GEMV copy
    prefill_bf16: int = 0     # bf16 copies for the prefill GEMMs
    kv: int = 0               # paged KV cache
    activations: int = 0      # decode + prefill activation buffers
    scratch: int = 0          # split-K, attention partials, collectives
    kv_pages: int = 0

    def items(self) -> dict[str, int]:
        return {k: v for k, v in dataclasses.asdict(self).items() if k != "kv_pages"}

    @property
    def total(self) -> int:
        return sum(self.items().values())


# KV precision tiers: bytes per stored K or V element (the scale of a block folded in)
KV_PRECISION_BYTES = {
    "bf16": 2.0,          # the engine's resident layout
    "fp8": 1.0 + 4 / 128,  # e4m3 codes + one f32 scale per (token, KV head) of 128 elements
    "q8": 34 / 32,         # q8_0 blocks: int8 codes + one f16 scale per 32 elements
}


def parse_kv_precision(s: str | None) -> str:
    """'' / None -> bf16; 'q8_0' is accepted for q8; anything else is refused (no silent default)."""
    t = (s or "bf16").lower()
    t = "q8" if t == "q8_0" else t
    if t not in KV_PRECISION_BYTES:
        raise ValueError(f"unknown KV precision {s!r} (want one of {sorted(KV_PRECISION_BYTES)})")
    return t


def kv_bytes_per_token(cfg: ModelConfig, tp: int = 1, precision: str = "bf16") -> int:
    """K and V of one token over all layers, for the KV heads one rank holds, at a KV precision tier.
    Span eviction re-rotates stored keys, so the lossy tiers (fp8, q8) cost accuracy at an eviction
    as well as at attention (the bf16 tier rounds once more per re-rotation)."""
    kv_heads = max(1, math.ceil(cfg.n_kv_heads / tp)) if cfg.n_kv_heads >= tp else 1
    elems = cfg.n_layers * 2 * kv_heads * cfg.head_dim
    return int(math.ceil(elems * KV_PRECISION_BYTES[parse_kv_precision(precision)]))


def select_kv_precision(cfg: ModelConfig, want_tokens: int, kv_budget_bytes: int, tp: int = 1) -> str:
    """The densest-needed tier: bf16 when ``want_tokens`` fit the KV budget in bf16, else the least
    lossy tier that fits (fp8, then q8 -- the same density order); raises when none fits."""
    for t in ("bf16", "fp8", "q8"):
        if want_tokens * kv_bytes_per_token(cfg, tp, t) <= kv_budget_bytes:
            return t
    raise ValueError(f"{want_tokens} tokens of KV do not fit {kv_budget_bytes / 2**30:.2f} GiB at any precision tier")


def weight_counts(cfg: ModelConfig, tp: int = 1, ep: int = 1) -> dict[str, int]:
    """Weights per rank by role (TP splits heads / FFN rows / vocab; EP splits the experts)."""
    d, L = cfg.d_model, cfg.n_layers
    q = cfg.n_heads * cfg.head_dim
    kv = cfg.n_kv_heads * cfg.head_dim
    attn_in = L * d * (q + 2 * kv) // tp
    # o_proj is row-parallel: a rank holds the 256-aligned column range around its heads
    attn_out = L * d * min(q, -(-(q // tp) // 256) * 256 + (256 if tp > 1 else 0))
    if cfg.is_moe:
        experts = L * -(-cfg.n_experts // max(ep, tp)) * 3 * d * cfg.expert_ffn_dim
        ffn = experts
    else:
        ffn = L * 3 * d * cfg.ffn_dim // tp
    lm = -(-cfg.vocab_size // tp) * d
    emb = cfg.vocab_size * d
    return {"attn_in": attn_in, "attn_out": attn_out, "ffn": ffn, "lm_head": lm, "embed": emb}


def plan(cfg: ModelConfig, mix: str = "q4_k_m", max_context: int = 8192, batch: int = 8, tp: int = 1, ep: int = 1,
         prefill_bf16: bool = True, max_prefill_tokens: int = 4096, kv_pages: int | None = None,
         kv_precision: str = "bf16") -> MemoryPlan:
    """Device bytes per rank of serving ``cfg`` with ``batch`` sequences of ``max_context`` tokens."""
    bpw = MIX_WEIGHT_BYTES.get(mix, BYTES_PER_WEIGHT.get(mix, 2.0))
    wc = weight_counts(cfg, tp, ep)
    linear = wc["attn_in"] + wc["attn_out"] + wc["ffn"] + wc["lm_head"]
    p = MemoryPlan()
    p.weights = int((linear + wc["embed"]) * bpw)
    dense_linear = linear - (wc["ffn"] if cfg.is_moe else 0)  # experts are not tile-packed / bf16-cached
    p.tile_packed = int(dense_linear * bpw)
    p.prefill_bf16 = int(dense_linear * 2) if prefill_bf16 else 0
    pages = kv_pages if kv_pages is not None else batch * -(-max_context // PAGE_TOKENS) + 1
    p.kv_pages = pages
    p.kv = pages * PAGE_TOKENS * kv_bytes_per_token(cfg, tp, kv_precision)
    d, f = cfg.d_model, (cfg.expert_ffn_dim * cfg.n_experts_used if cfg.is_moe else cfg.ffn_dim // tp)
    decode_act = batch * (4 * (d + 2 * f + cfg.vocab_size) + 2 * (d + f))
    prefill_act = max_prefill_tokens * (4 * 2 * d + 2 * (3 * d + 2 * f) + 4 * f)
    p.activations = decode_act + prefill_act
    p.scratch = 64 << 20  # split-K partials, attention partials, collective buffers (upper bound)
    return p


def check_fits(p: MemoryPlan, budget_bytes: int) -> MemoryPlan:
    if p.total > budget_bytes:
        raise FitError(p, budget_bytes)
    return p


def max_context(cfg: ModelConfig, budget_bytes: int, mix: str = "q4_k_m", batch: int = 8, tp: int = 1, ep: int = 1,
                prefill_bf16: bool = True) -> int:
    """Largest per-sequence context (a multiple of the page size) whose plan fits the budget."""
    base = plan(cfg, mix, PAGE_TOKENS, batch, tp, ep, prefill_bf16)
    free = budget_bytes - (base.total - base.kv)
    if free <= 0:
        raise FitError(base, budget_bytes)
    per_token = kv_bytes_per_token(cfg, tp) * batch
    ctx = (free // per_token) // PAGE_TOKENS * PAGE_TOKENS
    return int(min(ctx, cfg.max_context))


@dataclasses.dataclass(frozen=True)
class KVResidencySplit:
    """Placement of a KV cache over the device (hot: the span decode reads every step) and host
    memory (cold: the least recently attended span, spilled instead of evicted)."""
    hot_tokens: int
    cold_tokens: int
    bytes_per_token: int

    @property
    def tokens(self) -> int:
        return self.hot_tokens + self.cold_tokens

    @property
    def hot_bytes(self) -> int:
        return self.hot_tokens * self.bytes_per_token

    @property
    def cold_bytes(self) -> int:
        return self.cold_tokens * self.bytes_per_token


def kv_residency_split(want_tokens: int, bytes_per_token: int, device_free: int, host_free: int,
                       page_tokens: int = PAGE_TOKENS) -> KVResidencySplit:
    """How many of ``want_tokens`` stay on the device and how many spill to the host, given the
    free bytes of each pool.  Hot tokens fill whole pages of the device first; the rest spill to
    the host up to its room.  Fail-open: a non-positive want or per-token cost gives an empty
    split, and no host room gives the device-only sizing, so the effective context is never below
    device-only sizing.

    Reference: internal/compute/kvresidency.go (KVResidencySplit, the hot / cold policy)."""
    if want_tokens <= 0 or bytes_per_token <= 0:
        return KVResidencySplit(0, 0, max(0, bytes_per_token))
    page = page_tokens * bytes_per_token
    hot = min(want_tokens, max(0, device_free) // page * page_tokens)
    rest = want_tokens - hot
    cold = min(rest, max(0, host_free) // bytes_per_token) if rest > 0 else 0
    return KVResidencySplit(hot, cold, bytes_per_token)
