"""Rotary position embedding frequencies, with the context-extension scalings checkpoints declare.

``inv_freq(head_dim, theta, scaling, max_context)`` returns the per-pair inverse frequencies
(float64) and the attention scale folded into cos/sin:

* none     -- theta^(-2j/d);
* linear   -- positions interpolated by ``factor`` (every frequency / factor);
* dynamic  -- dynamic NTK: unchanged inside the trained context the tables cover;
* llama3   -- wavelength-banded interpolation: long wavelengths (> original / low_freq_factor) are
              divided by ``factor``, short ones (< original / high_freq_factor) kept, and the band in
              between blended linearly in original / wavelength;
* yarn     -- "YaRN" (Peng et al., 2023): dimensions whose rotation count over the original context
              lies between ``beta_slow`` and ``beta_fast`` blend linearly from interpolated
              (frequency / factor) to unchanged; cos/sin are scaled by m(factor, mscale) /
              m(factor, mscale_all_dim) with m(s, k) = 0.1 k ln(s) + 1 (plain m(s, 1) without them);
* longrope -- per-pair rescale factors (``long_factor`` when the table reaches past the original
              context, else ``short_factor``) and attention scale sqrt(1 + ln(s) / ln(original)).

The tables are static (built once for the engine's context), so the two length-dependent variants
(dynamic, longrope) are resolved for that context.

Reference: rope scaling / yarn / longrope helpers (internal/model/arch.go:26-180, longrope.go).
"""
from __future__ import annotations

import math

import torch


def _yarn_corr_dim(n_rot: float, dim: int, base: float, orig: int) -> float:
    """Pair index whose wavelength completes ``n_rot`` rotations over ``orig`` positions."""
    return dim * math.log(orig / (n_rot * 2 * math.pi)) / (2 * math.log(base))


def _mscale(factor: float, k: float = 1.0) -> float:
    return 0.1 * k * math.log(factor) + 1.0 if factor > 1 else 1.0


def inv_freq(head_dim: int, theta: float, scaling=None, max_context: int | None = None
             ) -> tuple[torch.Tensor, float]:
    """``scaling``: None, a dict, or the (key, value) pairs ``ModelConfig.rope_scaling`` holds."""
    if scaling is not None and not isinstance(scaling, dict):
        scaling = dict(scaling)
    half = head_dim // 2
    j = torch.arange(half, dtype=torch.float64)
    base = torch.pow(torch.tensor(theta, dtype=torch.float64), 2.0 * j / head_dim)
    inv = 1.0 / base
    if not scaling:
        return inv, 1.0
    kind = str(scaling.get("rope_type") or scaling.get("type") or "").lower()
    factor = float(scaling.get("factor", 1.0))
    if kind in ("", "default", "none", "dynamic"):
        return inv, 1.0
    if kind == "linear":
        return inv / factor, 1.0
    if kind == "llama3":
        orig = float(scaling.get("original_max_position_embeddings", 8192))
        lo, hi = float(scaling.get("low_freq_factor", 1.0)), float(scaling.get("high_freq_factor", 4.0))
        wl = 2 * math.pi / inv
        low_wl, high_wl = orig / lo, orig / hi
        smooth = (orig / wl - lo) / (hi - lo)
        blended = (1 - smooth) * inv / factor + smooth * inv
        out = torch.where(wl > low_wl, inv / factor, torch.where(wl < high_wl, inv, blended))
        return out, 1.0
    if kind == "yarn":
        orig = int(scaling.get("original_max_position_embeddings") or (max_context or 32768) / factor)
        beta_fast, beta_slow = float(scaling.get("beta_fast") or 32), float(scaling.get("beta_slow") or 1)
        low = _yarn_corr_dim(beta_fast, head_dim, theta, orig)
        high = _yarn_corr_dim(beta_slow, head_dim, theta, orig)
        if scaling.get("truncate", True):
            low, high = math.floor(low), math.ceil(high)
        low, high = max(low, 0), min(high, head_dim - 1)
        if low == high:
            high += 0.001
        ramp = torch.clamp((torch.arange(half, dtype=torch.float64) - low) / (high - low), 0, 1)
        out = (inv / factor) * ramp + inv * (1 - ramp)   # ramp 0: unchanged, 1: fully interpolated
        att = scaling.get("attention_factor")
        if att is None:
            ms, msa = scaling.get("mscale"), scaling.get("mscale_all_dim")
            att = _mscale(factor, float(ms)) / _mscale(factor, float(msa)) if ms and msa else _mscale(factor)
        return out, float(att)
    if kind == "longrope":
        orig = int(scaling.get("original_max_position_embeddings") or max_context or 4096)
        ctx = max_context or orig
        if "factor" not in scaling:
            factor = ctx / orig
        ext = scaling["long_factor"] if ctx > orig else scaling["short_factor"]
        ext = torch.tensor(list(ext), dtype=torch.float64)
        att = scaling.get("attention_factor")
        if att is None:
            att = math.sqrt(1 + math.log(factor) / math.log(orig)) if factor > 1 else 1.0
        return 1.0 / (ext * base), float(att)
    raise ValueError(f"unsupported rope scaling {kind!r}")


def cos_sin(positions: torch.Tensor, head_dim: int, theta: float, scaling=None, max_context: int | None = None
            ) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 cos/sin [T, head_dim/2] with angles evaluated in float64 (times the attention scale)."""
    inv, m = inv_freq(head_dim, theta, scaling, max_context)
    ang = positions.to(torch.float64).cpu()[:, None] * inv[None, :]
    return (torch.cos(ang) * m).float(), (torch.sin(ang) * m).float()
