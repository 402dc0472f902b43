"""Roofline / cost model of decode and prefill on the measured peaks of the GPU.

Denominators come from ``MEASURED_PEAKS.json`` next to the repository root when present (a
STREAM-style copy bandwidth and a cuBLAS bf16 GEMM, burst and sustained), else from nominal B200
figures; every fraction this module reports names which one it used.

* ``decode_step``: bytes one decode step must move (every weight once, plus the KV of every
  sequence, with shared-prefix pages counted once when they fit in L2) and FLOPs;
  ``time_s`` = max(bytes / HBM, flops / tensor peak).
* ``prefill``: FLOPs of a prefill chunk (linear layers + causal attention over the cached prefix).
* ``collective``: bytes a tensor-parallel step must cross NVLink, for the fused-collective roofline
  (the slower of its compute at peak and its bytes at the measured link bandwidth).
* ``fraction(achieved, roof)``: achieved / roofline.

Reference: PrefillCostModel / PredictTime (internal/compute/prefill.go:47-300), decode roofline
(internal/model/decode_roofline.go), FusionTraffic (internal/compute/fusion_traffic.go:38-166).
"""
from __future__ import annotations

import dataclasses
import json
import os

from ..capacity import MIX_WEIGHT_BYTES, kv_bytes_per_token, weight_counts
from ..config import ModelConfig

NOMINAL = {"hbm_gbs": 7700.0, "bf16_tflops": 2250.0, "bf16_tflops_sustained": 2250.0, "nvlink_gbs": 900.0,
           "l2_bytes": 126 * 2**20, "source": "nominal B200"}
MEASURED_NVLINK_GBS = 770.0  # peer copy per direction per GPU on this pool


@dataclasses.dataclass
class Peaks:
    hbm_gbs: float
    bf16_tflops: float
    bf16_tflops_sustained: float
    nvlink_gbs: float
    l2_bytes: int
    source: str


def load_peaks(path: str | None = None) -> Peaks:
    """MEASURED_PEAKS.json (repository root, or ``path``) if present, else nominal figures."""
    if path is None:
        path = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                            "MEASURED_PEAKS.json")
    d = dict(NOMINAL)
    if os.path.exists(path):
        with open(path) as f:
            m = json.load(f)
        for k in ("hbm_gbs", "bf16_tflops", "bf16_tflops_sustained"):
            if k in m:
                d[k] = float(m[k])
        d["nvlink_gbs"] = MEASURED_NVLINK_GBS
        d["source"] = "measured"
    return Peaks(d["hbm_gbs"], d["bf16_tflops"], d["bf16_tflops_sustained"], d["nvlink_gbs"], int(d["l2_bytes"]),
                 d["source"])


@dataclasses.dataclass
class Roof:
    bytes: float
    flops: float
    time_s: float
    bound: str        # "memory" | "compute" | "link"
    source: str


def _roof(nbytes: float, flops: float, peaks: Peaks, sustained: bool = True, link_bytes: float = 0.0) -> Roof:
    tf = peaks.bf16_tflops_sustained if sustained else peaks.bf16_tflops
    t_mem = nbytes / (peaks.hbm_gbs * 1e9)
    t_cmp = flops / (tf * 1e12)
    t_lnk = link_bytes / (peaks.nvlink_gbs * 1e9)
    t = max(t_mem, t_cmp, t_lnk)
    bound = "memory" if t == t_mem else ("compute" if t == t_cmp else "link")
    return Roof(nbytes, flops, t, bound, peaks.source)


def decode_step(cfg: ModelConfig, batch: int, ctx: int, mix: str = "q4_k_m", tp: int = 1, ep: int = 1,
                shared_prefix: int = 0, peaks: Peaks | None = None) -> Roof:
    """Roofline of one decode step per rank: ``batch`` sequences at context ``ctx`` of which the first
    ``shared_prefix`` tokens are the same pages for all sequences."""
    peaks = peaks or load_peaks()
    bpw = MIX_WEIGHT_BYTES.get(mix, 2.0)
    wc = weight_counts(cfg, tp, ep)
    if cfg.is_moe:
        # only the routed experts of the batch are read (at most all local experts)
        per_expert = 3 * cfg.d_model * cfg.expert_ffn_dim * cfg.n_layers
        local = -(-cfg.n_experts // max(ep, tp))
        wc["ffn"] = min(local, batch * cfg.n_experts_used) * per_expert
    w_bytes = (wc["attn_in"] + wc["attn_out"] + wc["ffn"] + wc["lm_head"]) * bpw
    kv_tok = kv_bytes_per_token(cfg, tp)
    private = max(0, ctx - shared_prefix)
    shared_once = shared_prefix * kv_tok
    kv_bytes = batch * private * kv_tok + (shared_once if batch > 1 else shared_prefix * kv_tok)
    if batch > 1 and shared_once / cfg.n_layers > peaks.l2_bytes:  # one layer's prefix does not fit L2
        kv_bytes += (batch - 1) * shared_once
    flops = 2.0 * batch * (w_bytes / bpw) + 4.0 * batch * ctx * cfg.n_heads // tp * cfg.head_dim * cfg.n_layers
    return _roof(w_bytes + kv_bytes, flops, peaks)


def prefill(cfg: ModelConfig, tokens: int, cached: int = 0, tp: int = 1, peaks: Peaks | None = None) -> Roof:
    """Roofline of prefilling ``tokens`` new tokens after ``cached`` tokens already in the KV cache
    (bf16 weights; attention over the prefix plus the causal chunk)."""
    peaks = peaks or load_peaks()
    wc = weight_counts(cfg, tp)
    if cfg.is_moe:
        wc["ffn"] = cfg.n_layers * cfg.n_experts_used * 3 * cfg.d_model * cfg.expert_ffn_dim
    linear = wc["attn_in"] + wc["attn_out"] + wc["ffn"]
    attn_ctx = cached * tokens + tokens * (tokens + 1) / 2
    flops = 2.0 * tokens * linear + 4.0 * attn_ctx * cfg.n_heads // tp * cfg.head_dim * cfg.n_layers
    nbytes = linear * 2 + tokens * (cached + tokens) / max(1, tokens) * kv_bytes_per_token(cfg, tp)
    return _roof(nbytes, flops, peaks)


def collective(cfg: ModelConfig, batch: int, tp: int, peaks: Peaks | None = None) -> Roof:
    """Bytes one decode step sends over NVLink per rank under head-parallel attention (gather of the
    int8 attention output) and a K-split FFN (all-reduce of the fp32 residual)."""
    peaks = peaks or load_peaks()
    if tp <= 1:
        return _roof(0.0, 0.0, peaks)
    gather = batch * cfg.q_dim * (1 + 1 / 16) * (tp - 1) / tp          # int8 + per-32 (scale, sum)
    reduce = batch * cfg.d_model * 4 * 2 * (tp - 1) / tp                 # reduce-scatter + all-gather
    link = cfg.n_layers * (gather + reduce)
    return _roof(0.0, 0.0, peaks, link_bytes=link)


def fraction(achieved_s: float, roof: Roof) -> float:
    """roofline time / achieved time (1.0 = at the roofline)."""
    return roof.time_s / achieved_s if achieved_s > 0 else 0.0
