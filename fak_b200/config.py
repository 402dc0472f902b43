"""Model and engine configuration.

``ModelConfig`` covers the decoder families the engine runs: Llama (SmolLM2),
Qwen2 (qkv bias), Qwen3 (qk-norm) and Qwen3-MoE (softmax top-k router).  It is
built from GGUF metadata the same way the reference derives its
``model.Config`` (internal/model/config.go:374-605, internal/ggufload/gguf_config.go)
or from one of the named presets used by the benchmarks.

``EngineConfig`` is the single typed place for runtime knobs; every field can
be overridden by a ``FAK_*`` environment variable (the reference scatters
~100 such knobs across packages, e.g. FAK_CUDA_GRAPH, FAK_PAGED_KV_BLOCK_TOKENS,
FAK_NATIVE_MAX_RUNNING, FAK_INKERNEL_RADIX_BUDGET).
"""
from __future__ import annotations

import dataclasses
import os
from typing import Any


@dataclasses.dataclass(frozen=True)
class ModelConfig:
    arch: str  # "llama" | "qwen2" | "qwen3" | "qwen3moe" | "gemma2"
    n_layers: int
    d_model: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    ffn_dim: int
    vocab_size: int
    rms_eps: float = 1e-5
    rope_theta: float = 10000.0
    tie_embeddings: bool = False
    qkv_bias: bool = False
    qk_norm: bool = False
    n_experts: int = 0
    n_experts_used: int = 0
    expert_ffn_dim: int = 0
    norm_topk_prob: bool = True
    max_context: int = 32768
    # context-extension RoPE scaling as sorted (key, value) pairs (hashable; a dict is accepted):
    # type linear|yarn|llama3, factor, original_max_position_embeddings, beta_fast/slow, ...
    rope_scaling: tuple | None = None
    # sliding-window attention: each query sees the last ``sliding_window`` keys (0 = full causal)
    # on the layers in ``swa_layers`` (None = every layer)
    sliding_window: int = 0
    swa_layers: tuple | None = None
    # Gemma-style blocks: gated activation ("silu" or "gelu_tanh"), score / logit soft-capping
    # (cap * tanh(x / cap); 0 = none), sandwich norms (a norm after attention and after the FFN,
    # before each residual add), embedding scale, attention scale (0 = 1/sqrt(head_dim))
    act: str = "silu"
    attn_softcap: float = 0.0
    final_softcap: float = 0.0
    sandwich_norms: bool = False
    embed_scale: float = 1.0
    attn_scale: float = 0.0
    # gpt-oss blocks: a learned per-head sink logit in every attention softmax (``attn_sinks``),
    # an output-projection bias, a biased router that keeps the top-k logits and then takes the
    # softmax over those k (``router`` "topk_softmax"; default "softmax_topk" = softmax over all
    # experts, then top-k), biased experts, and the clamped OAI gate
    # (up + 1) * g * sigmoid(alpha * g) with g <= limit, |up| <= limit (``swiglu_alpha`` > 0)
    attn_sinks: bool = False
    attn_out_bias: bool = False
    router: str = "softmax_topk"
    moe_bias: bool = False
    swiglu_alpha: float = 0.0
    swiglu_limit: float = 0.0
    # Qwen3.5 hybrid blocks: the layers in ``linear_layers`` mix tokens with a gated delta rule
    # (Gated DeltaNet: causal depthwise conv of width ``gdn_conv``, ``gdn_k_heads`` key heads of
    # ``gdn_k_dim``, ``gdn_v_heads`` value heads of ``gdn_v_dim``, a decayed key-value state per
    # head) instead of softmax attention; full-attention layers gate their output per channel with
    # sigmoid(gate) from a doubled q projection (``attn_out_gate``) and rotate only the first
    # ``rotary_dim`` dims of each head (0 = all)
    linear_layers: tuple | None = None
    gdn_conv: int = 4
    gdn_k_heads: int = 0
    gdn_v_heads: int = 0
    gdn_k_dim: int = 0
    gdn_v_dim: int = 0
    attn_out_gate: bool = False
    rotary_dim: int = 0
    bos_token_id: int = 1
    eos_token_id: int = 2
    name: str = ""

    @property
    def q_dim(self) -> int:
        return self.n_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    @property
    def gqa_group(self) -> int:
        return self.n_heads // self.n_kv_heads

    @property
    def is_moe(self) -> bool:
        return self.n_experts > 0

    def __post_init__(self) -> None:
        if isinstance(self.rope_scaling, dict):
            items = ((k, tuple(v) if isinstance(v, list) else v) for k, v in self.rope_scaling.items())
            object.__setattr__(self, "rope_scaling", tuple(sorted(items)) or None)

    def is_linear(self, i: int) -> bool:
        return self.linear_layers is not None and i in self.linear_layers

    @property
    def rope_dim(self) -> int:
        return self.rotary_dim or self.head_dim

    def device_gap(self) -> str | None:
        """Why the device engine cannot run this config (None when it can).  Such models run on the
        fp32 reference model (``models.reference.ReferenceModel``)."""
        if self.swiglu_alpha and (abs(self.swiglu_alpha - 1.702) > 1e-6 or abs(self.swiglu_limit - 7.0) > 1e-6):
            return "the device's clamped gate is gpt-oss's (alpha 1.702, limit 7)"
        if (self.attn_sinks or self.moe_bias or self.swiglu_alpha) and self.head_dim not in (64, 128):
            return "gpt-oss blocks on the device need head dim 64 or 128"
        if self.linear_layers or self.attn_out_gate or (self.rotary_dim and self.rotary_dim != self.head_dim):
            return "Qwen3.5 hybrid blocks (Gated DeltaNet layers, gated partial-rotary attention) have no device kernels"
        return None

    def layer_window(self, i: int) -> int:
        if self.sliding_window <= 0:
            return 0
        return self.sliding_window if self.swa_layers is None or i in self.swa_layers else 0

    def max_window(self) -> int:
        """The widest window when EVERY layer is windowed (keys older than it are never read
        again), else 0."""
        ws = [self.layer_window(i) for i in range(self.n_layers)]
        return max(ws) if ws and min(ws) > 0 else 0

    def validate(self) -> None:
        if self.n_heads % self.n_kv_heads:
            raise ValueError(f"n_heads {self.n_heads} not a multiple of n_kv_heads {self.n_kv_heads}")
        if self.head_dim % 2:
            raise ValueError("head_dim must be even for RoPE")
        if self.is_moe and not (0 < self.n_experts_used <= self.n_experts):
            raise ValueError("MoE config needs 0 < n_experts_used <= n_experts")
        if self.router not in ("softmax_topk", "topk_softmax"):
            raise ValueError(f"unknown router {self.router!r}")

    def param_count(self) -> int:
        d, L = self.d_model, self.n_layers
        attn = d * self.q_dim + 2 * d * self.kv_dim + self.q_dim * d
        if self.is_moe:
            ffn = self.n_experts * 3 * d * self.expert_ffn_dim + d * self.n_experts
        else:
            ffn = 3 * d * self.ffn_dim
        emb = self.vocab_size * d * (1 if self.tie_embeddings else 2)
        return L * (attn + ffn) + emb

    def replace(self, **kw: Any) -> "ModelConfig":
        return dataclasses.replace(self, **kw)


PRESETS: dict[str, ModelConfig] = {
    # SmolLM2-135M (HF config): 30 layers, 576 wide, 9/3 heads of 64, FFN 1536, tied, theta 1e4
    "smollm2-135m": ModelConfig("llama", 30, 576, 9, 3, 64, 1536, 49152, 1e-5, 10000.0, tie_embeddings=True,
                                max_context=8192, bos_token_id=1, eos_token_id=2, name="smollm2-135m"),
    # Qwen2.5-7B: 28 layers, 3584 wide, 28/4 heads of 128, FFN 18944, qkv bias, theta 1e6
    "qwen2.5-7b": ModelConfig("qwen2", 28, 3584, 28, 4, 128, 18944, 152064, 1e-6, 1e6, qkv_bias=True,
                              max_context=32768, bos_token_id=151643, eos_token_id=151645, name="qwen2.5-7b"),
    # Qwen2.5-32B: 64 layers, 5120 wide, 40/8 heads of 128, FFN 27648
    "qwen2.5-32b": ModelConfig("qwen2", 64, 5120, 40, 8, 128, 27648, 152064, 1e-6, 1e6, qkv_bias=True,
                               max_context=32768, bos_token_id=151643, eos_token_id=151645, name="qwen2.5-32b"),
    # Qwen3-30B-A3B: 48 layers, 2048 wide, 32/4 heads of 128, 128 experts top-8, expert FFN 768, qk-norm
    "qwen3-30b-a3b": ModelConfig("qwen3moe", 48, 2048, 32, 4, 128, 6144, 151936, 1e-6, 1e6, qk_norm=True,
                                 n_experts=128, n_experts_used=8, expert_ffn_dim=768, norm_topk_prob=True,
                                 max_context=32768, bos_token_id=151643, eos_token_id=151645,
                                 name="qwen3-30b-a3b"),
    # gpt-oss-20b: 24 layers, 2880 wide, 64/8 heads of 64, 32 experts top-4 of width 2880 (MXFP4 in
    # the checkpoint), attention sinks, biases everywhere, 128-token windows on the even layers,
    # YaRN x32 over a 4096-token original context, theta 150000
    "gpt-oss-20b": ModelConfig("gptoss", 24, 2880, 64, 8, 64, 2880, 201088, 1e-5, 150000.0, qkv_bias=True,
                               n_experts=32, n_experts_used=4, expert_ffn_dim=2880, max_context=131072,
                               rope_scaling={"type": "yarn", "factor": 32.0, "beta_fast": 32.0, "beta_slow": 1.0,
                                             "original_max_position_embeddings": 4096, "truncate": False},
                               sliding_window=128, swa_layers=tuple(range(0, 24, 2)), attn_sinks=True,
                               attn_out_bias=True, router="topk_softmax", moe_bias=True, swiglu_alpha=1.702,
                               swiglu_limit=7.0, bos_token_id=199998, eos_token_id=200002, name="gpt-oss-20b"),
    # small shapes for tests (same structure, few layers)
    "tiny-llama": ModelConfig("llama", 2, 256, 4, 2, 64, 512, 512, 1e-5, 10000.0, tie_embeddings=True,
                              max_context=1024, name="tiny-llama"),
    "tiny-qwen2": ModelConfig("qwen2", 2, 512, 8, 2, 64, 1024, 1024, 1e-6, 1e6, qkv_bias=True,
                              max_context=2048, name="tiny-qwen2"),
    # Gemma-2 shaped test model: GELU-tanh FFN, sandwich norms, soft-capping, alternating windows
    "tiny-gemma2": ModelConfig("gemma2", 2, 256, 4, 2, 64, 512, 512, 1e-6, 1e4, tie_embeddings=True,
                               act="gelu_tanh", attn_softcap=50.0, final_softcap=30.0, sandwich_norms=True,
                               embed_scale=16.0, sliding_window=32, swa_layers=(0,), max_context=1024,
                               name="tiny-gemma2"),
    "tiny-gptoss": ModelConfig("gptoss", 2, 256, 4, 2, 64, 256, 512, 1e-5, 150000.0, qkv_bias=True,
                               n_experts=4, n_experts_used=2, expert_ffn_dim=128, max_context=2048,
                               rope_scaling={"type": "yarn", "factor": 32.0, "beta_fast": 32.0, "beta_slow": 1.0,
                                             "original_max_position_embeddings": 64, "truncate": False},
                               sliding_window=16, swa_layers=(0,), attn_sinks=True, attn_out_bias=True,
                               router="topk_softmax", moe_bias=True, swiglu_alpha=1.702, swiglu_limit=7.0,
                               name="tiny-gptoss"),
    "tiny-qwen3moe": ModelConfig("qwen3moe", 2, 512, 8, 2, 64, 1024, 1024, 1e-6, 1e6, qk_norm=True,
                                 n_experts=8, n_experts_used=2, expert_ffn_dim=256, max_context=2048,
                                 name="tiny-qwen3moe"),
}


def preset(name: str) -> ModelConfig:
    try:
        return PRESETS[name]
    except KeyError as e:
        raise KeyError(f"unknown model preset {name!r}; known: {sorted(PRESETS)}") from e


def config_from_gguf_metadata(meta: dict[str, Any], tensor_shapes: dict[str, tuple[int, ...]] | None = None
                              ) -> ModelConfig:
    """Derive a ModelConfig from GGUF metadata (keys ``{arch}.*`` as written by llama.cpp)."""
    arch = meta.get("general.architecture")
    if arch not in ("llama", "qwen2", "qwen3", "qwen3moe", "mistral", "gemma2"):
        raise ValueError(f"unsupported GGUF architecture {arch!r}")

    def g(key: str, default: Any = None) -> Any:
        return meta.get(f"{arch}.{key}", default)

    d = int(g("embedding_length"))
    nh = int(g("attention.head_count"))
    nkv = int(g("attention.head_count_kv", nh))
    hd = int(g("attention.key_length", d // nh))
    vocab = g("vocab_size")
    shapes = tensor_shapes or {}
    if vocab is None:
        toks = meta.get("tokenizer.ggml.tokens")
        vocab = len(toks) if toks else shapes.get("token_embd.weight", (0,))[0]
    tied = "output.weight" not in shapes if shapes else bool(meta.get("fak.tie_embeddings", False))
    qkv_bias = "blk.0.attn_q.bias" in shapes if shapes else arch == "qwen2"
    qk_norm = "blk.0.attn_q_norm.weight" in shapes if shapes else arch.startswith("qwen3")
    n_exp = int(g("expert_count", 0) or 0)
    cfg = ModelConfig(
        arch="llama" if arch == "mistral" else arch,
        n_layers=int(g("block_count")),
        d_model=d,
        n_heads=nh,
        n_kv_heads=nkv,
        head_dim=hd,
        ffn_dim=int(g("feed_forward_length", 0) or 0),
        vocab_size=int(vocab),
        rms_eps=float(f"{float(g('attention.layer_norm_rms_epsilon', 1e-5)):.6g}"),
        rope_theta=float(f"{float(g('rope.freq_base', 10000.0)):.7g}"),
        rope_scaling=_gguf_rope_scaling(g),
        sliding_window=int(g("attention.sliding_window", 0) or 0),
        tie_embeddings=tied,
        qkv_bias=qkv_bias,
        qk_norm=qk_norm,
        n_experts=n_exp,
        n_experts_used=int(g("expert_used_count", 0) or 0),
        expert_ffn_dim=int(g("expert_feed_forward_length", 0) or 0),
        norm_topk_prob=bool(g("expert_weights_norm", True)),
        max_context=int(g("context_length", 4096)),
        bos_token_id=int(meta.get("tokenizer.ggml.bos_token_id", 1)),
        eos_token_id=int(meta.get("tokenizer.ggml.eos_token_id", 2)),
        name=str(meta.get("general.name", "")),
    )
    if arch == "gemma2":   # GELU-tanh FFN, sandwich norms, soft-capping, every other layer windowed
        cfg = cfg.replace(act="gelu_tanh", sandwich_norms=True, embed_scale=float(d) ** 0.5,
                          attn_softcap=float(g("attn_logit_softcapping", 50.0) or 0.0),
                          final_softcap=float(g("final_logit_softcapping", 30.0) or 0.0),
                          sliding_window=int(g("attention.sliding_window", 4096) or 0),
                          swa_layers=tuple(range(0, cfg.n_layers, 2)))
    cfg.validate()
    return cfg


def _gguf_rope_scaling(g) -> dict | None:
    """``{arch}.rope.scaling.*`` keys (type, factor, original_context_length, yarn betas/log-mul)."""
    kind = str(g("rope.scaling.type", "") or "").lower()
    factor = float(g("rope.scaling.factor", 0.0) or 0.0)
    if kind in ("", "none") or factor in (0.0, 1.0):
        return None
    out: dict[str, Any] = {"type": kind, "factor": factor}
    orig = g("rope.scaling.original_context_length", None)
    if orig:
        out["original_max_position_embeddings"] = int(orig)
    for src, dst in (("rope.scaling.yarn_beta_fast", "beta_fast"), ("rope.scaling.yarn_beta_slow", "beta_slow")):
        v = g(src, None)
        if v is not None:
            out[dst] = float(v)
    return out


def _env(name: str, default: Any, typ: type) -> Any:
    v = os.environ.get(name)
    if v is None or v == "":
        return default
    if typ is bool:
        return v.lower() in ("1", "true", "yes", "on")
    return typ(v)


@dataclasses.dataclass
class EngineConfig:
    """Runtime knobs (each one overridable by the FAK_* variable named in ENV_KEYS)."""
    page_size: int = 16                 # tokens per KV page
    kv_pages: int = 0                   # 0: size from free memory * kv_mem_fraction
    kv_mem_fraction: float = 0.5
    max_batch: int = 64                 # max running decode lanes
    max_prefill_tokens: int = 4096      # chunked-prefill chunk
    cuda_graph: bool = True
    graph_batch_buckets: tuple[int, ...] = (1, 2, 4, 8, 16, 32, 64)
    radix_cache: bool = True
    radix_budget_pages: int = 0         # 0: unlimited (evict only under KV pressure)
    tp: int = 1
    ep: int = 1
    fused_collectives: bool = True      # in-kernel P2P collectives; False = NCCL baseline
    prefill_bf16_weights: bool = True   # keep a bf16 copy of each quantized weight for prefill GEMMs
    seed: int = 0
    spec_k: int = 0                     # draft tokens per verify step (0: no speculation)
    spec_draft_layers: int = 4          # self-speculation: the draft is the first N layers + LM head
    spec_drafter: str = "self"          # self | lookup | multi (self vs lookup by acceptance) | tree (lookup tree)
    spec_tree_width: int = 3            # tree speculation: continuations (branches) per round
    fused_activations: bool = False     # decode GEMVs normalise+quantize fp32 inputs themselves
    attention_merge: bool = False       # merge attention splits in the last split's CTA (no combine launch)
    l2_prefetch: bool = False           # decode kernels warm L2 with the next GEMV's weights (measured neutral)
    cascade_attention: bool = False     # decode: a batch's shared prefix pages attended once for all lanes
                                        # (measured: no faster than the split-KV path yet at 5 lanes x 9K)
    debug_poison: bool = False          # fill scratch with NaN and the KV cache with a large sentinel at start
                                        # (a kernel reading memory nobody wrote shows up in its outputs)
    preempt_mode: str = "recompute"     # out of KV pages: "recompute" (radix-assisted) or "swap" to host memory
    swap_space_gb: float = 16.0         # pinned host memory for swapped-out KV pages
    async_decode: bool = True           # device-resident lane state; tokens read back one step behind
    p2p_spin_limit: int = 0             # polls before a cross-rank wait gives up (0: kernel default, ~1 s)
    cpu_offload_experts: bool = False   # MoE experts in host memory, their FFNs on the CPU (no CUDA graphs)

    ENV_KEYS = {
        "page_size": ("FAK_PAGED_KV_BLOCK_TOKENS", int),
        "kv_pages": ("FAK_KV_PAGES", int),
        "kv_mem_fraction": ("FAK_KV_MEM_FRACTION", float),
        "max_batch": ("FAK_NATIVE_MAX_RUNNING", int),
        "max_prefill_tokens": ("FAK_MAX_PREFILL_TOKENS", int),
        "cuda_graph": ("FAK_CUDA_GRAPH", bool),
        "radix_cache": ("FAK_INKERNEL_RADIX", bool),
        "radix_budget_pages": ("FAK_INKERNEL_RADIX_BUDGET", int),
        "tp": ("FAK_TENSOR_PARALLEL", int),
        "ep": ("FAK_EXPERT_PARALLEL", int),
        "fused_collectives": ("FAK_FUSED_COLLECTIVES", bool),
        "prefill_bf16_weights": ("FAK_PREFILL_BF16", bool),
        "seed": ("FAK_SEED", int),
        "spec_k": ("FAK_SPEC_K", int),
        "spec_draft_layers": ("FAK_SPEC_DRAFT_LAYERS", int),
        "spec_drafter": ("FAK_SPEC_DRAFTER", str),
        "spec_tree_width": ("FAK_SPEC_TREE_WIDTH", int),
        "fused_activations": ("FAK_FUSED_ACT", bool),
        "attention_merge": ("FAK_ATTN_MERGE", bool),
        "l2_prefetch": ("FAK_L2_PREFETCH", bool),
        "cascade_attention": ("FAK_CASCADE_ATTN", bool),
        "debug_poison": ("FAK_DEBUG_POISON", bool),
        "preempt_mode": ("FAK_PREEMPT_MODE", str),
        "swap_space_gb": ("FAK_SWAP_SPACE_GB", float),
        "async_decode": ("FAK_ASYNC_DECODE", bool),
        "p2p_spin_limit": ("FAK_P2P_SPIN_LIMIT", int),
        "cpu_offload_experts": ("FAK_CPU_OFFLOAD_EXPERTS", bool),
    }

    @classmethod
    def from_env(cls, **overrides: Any) -> "EngineConfig":
        cfg = cls(**overrides)
        for fname, (env, typ) in cls.ENV_KEYS.items():
            if fname in overrides:
                continue
            setattr(cfg, fname, _env(env, getattr(cfg, fname), typ))
        return cfg
