"""Gemma-4 dense text decoders on the fp32 reference path.

Gemma-4 interleaves two attention regimes with different shapes per layer:

* sliding layers: ``head_dim`` wide heads, ``num_key_value_heads`` KV heads, a ``sliding_window``
  causal window and their own RoPE base;
* full layers: ``global_head_dim`` wide heads; with ``attention_k_eq_v`` a single projection
  (``num_global_key_value_heads`` heads) serves as both key and value (no v_proj); "proportional"
  RoPE rotates only the first ``partial_rotary_factor`` of the frequencies (the rest stay at angle 0).

Every layer RMS-normalises q and k per head with a learned gain and v per head without one, uses a
softmax scale of exactly 1, wraps attention and FFN in sandwich norms (plain ``w`` gains), and
multiplies the block output by a learned per-layer scalar.  Embeddings are scaled by
sqrt(hidden_size); the FFN is GELU-tanh gated; logits are soft-capped when
``final_logit_softcapping`` is set.

The model reads a Hugging Face checkpoint (config.json + safetensors) and runs whole sequences.
Per-layer input embeddings, the MoE block and KV-shared layers (options of some Gemma-4 configs)
are refused.

Reference: internal/model/gemma4.go (per-layer geometry, k-as-v global layers, q/k/v norms, scale
1, sandwich norms, layer output scale), internal/model/gemma4_invfreq.go (the global layers'
frequency vector).
"""
from __future__ import annotations

import glob
import json
import math
import os

import torch

from .hf import _to_f32, read_safetensors


def _norm(x: torch.Tensor, w: torch.Tensor | None, eps: float) -> torch.Tensor:
    y = x * torch.pow(x.pow(2).mean(-1, keepdim=True) + eps, -0.5)
    return y * w if w is not None else y


def _inv_freq(rp: dict, head_dim: int) -> torch.Tensor:
    """Inverse frequencies [head_dim / 2] of one layer type ("default" or "proportional")."""
    kind = rp.get("rope_type", "default")
    base = float(rp["rope_theta"])
    j = torch.arange(0, head_dim, 2, dtype=torch.float64)
    if kind == "default":
        return 1.0 / base ** (j / head_dim)
    if kind == "proportional":
        n_rot = int(float(rp.get("partial_rotary_factor", 1.0)) * head_dim // 2)
        inv = torch.zeros(head_dim // 2, dtype=torch.float64)
        inv[:n_rot] = 1.0 / base ** (j[:n_rot] / head_dim)
        return inv / float(rp.get("factor", 1.0))
    raise ValueError(f"unsupported Gemma-4 rope type {kind!r}")


def _rope(x: torch.Tensor, inv: torch.Tensor) -> torch.Tensor:
    """rotate-half RoPE of x [T, H, D] at positions 0..T-1."""
    T, D = x.shape[0], x.shape[-1]
    ang = torch.arange(T, dtype=torch.float64)[:, None] * inv[None, :]
    c, s = torch.cos(ang).float()[:, None, :], torch.sin(ang).float()[:, None, :]
    x0, x1 = x[..., :D // 2], x[..., D // 2:]
    return torch.cat([x0 * c - x1 * s, x1 * c + x0 * s], dim=-1)


class Gemma4Reference:
    def __init__(self, hf: dict, tensors: dict[str, torch.Tensor]):
        c = hf.get("text_config") if isinstance(hf.get("text_config"), dict) else hf
        if c.get("hidden_size_per_layer_input"):
            raise NotImplementedError("Gemma-4 per-layer input embeddings are not supported")
        if c.get("enable_moe_block"):
            raise NotImplementedError("the Gemma-4 MoE block is not supported")
        if int(c.get("num_kv_shared_layers") or 0):
            raise NotImplementedError("Gemma-4 KV-shared layers are not supported")
        self.c = c
        prefix = "model.language_model." if any(k.startswith("model.language_model.") for k in tensors) else "model."
        self.t = {k[len(prefix):] if k.startswith(prefix) else k: v.float() for k, v in tensors.items()}
        self.eps = float(c.get("rms_norm_eps", 1e-6))
        self.types = list(c["layer_types"])
        self.inv = {lt: _inv_freq(c["rope_parameters"][lt],
                                  int(c["global_head_dim"]) if lt == "full_attention" and c.get("global_head_dim")
                                  and c["rope_parameters"][lt].get("rope_type") == "proportional" else int(c["head_dim"]))
                    for lt in set(self.types)}

    @classmethod
    def from_hf(cls, model_dir: str) -> "Gemma4Reference":
        with open(os.path.join(model_dir, "config.json")) as f:
            hf = json.load(f)
        t = {}
        for p in sorted(glob.glob(os.path.join(model_dir, "*.safetensors"))):
            for n, (dt, shape, arr) in read_safetensors(p).items():
                t[n] = torch.from_numpy(_to_f32(dt, arr).reshape(shape).copy())
        return cls(hf, t)

    def w(self, n: str) -> torch.Tensor:
        return self.t[n]

    def attention(self, i: int, x: torch.Tensor) -> torch.Tensor:
        c, p = self.c, f"layers.{i}.self_attn."
        T = x.shape[0]
        full = self.types[i] == "full_attention"
        D = int(c["global_head_dim"]) if full and c.get("global_head_dim") else int(c["head_dim"])
        k_eq_v = bool(c.get("attention_k_eq_v")) and full
        H = int(c["num_attention_heads"])
        q = _norm((x @ self.w(p + "q_proj.weight").T).view(T, H, D), self.w(p + "q_norm.weight"), self.eps)
        kraw = (x @ self.w(p + "k_proj.weight").T).view(T, -1, D)
        vraw = kraw if k_eq_v else (x @ self.w(p + "v_proj.weight").T).view(T, -1, D)
        k = _norm(kraw, self.w(p + "k_norm.weight"), self.eps)
        v = _norm(vraw, None, self.eps)
        inv = self.inv[self.types[i]]
        q, k = _rope(q, inv), _rope(k, inv)
        g = H // k.shape[1]
        k, v = k.repeat_interleave(g, dim=1), v.repeat_interleave(g, dim=1)
        s = torch.einsum("thd,khd->htk", q, k)                      # softmax scale 1
        qpos, kpos = torch.arange(T)[:, None], torch.arange(T)[None, :]
        masked = kpos > qpos
        if not full and c.get("sliding_window"):
            masked |= kpos <= qpos - int(c["sliding_window"])
        s = s.masked_fill(masked[None], -math.inf)
        o = torch.einsum("htk,khd->thd", torch.softmax(s, -1), v).reshape(T, H * D)
        return o @ self.w(p + "o_proj.weight").T

    @torch.no_grad()
    def forward(self, ids) -> torch.Tensor:
        c = self.c
        ids = torch.as_tensor(ids, dtype=torch.long).reshape(-1)
        emb = self.w("embed_tokens.weight")
        x = emb[ids] * torch.tensor(float(c["hidden_size"]) ** 0.5, dtype=torch.float32)
        for i in range(int(c["num_hidden_layers"])):
            p = f"layers.{i}."
            a = self.attention(i, _norm(x, self.w(p + "input_layernorm.weight"), self.eps))
            x = x + _norm(a, self.w(p + "post_attention_layernorm.weight"), self.eps)
            h = _norm(x, self.w(p + "pre_feedforward_layernorm.weight"), self.eps)
            g = h @ self.w(p + "mlp.gate_proj.weight").T
            u = h @ self.w(p + "mlp.up_proj.weight").T
            f = (torch.nn.functional.gelu(g, approximate="tanh") * u) @ self.w(p + "mlp.down_proj.weight").T
            x = x + _norm(f, self.w(p + "post_feedforward_layernorm.weight"), self.eps)
            if p + "layer_scalar" in self.t:
                x = x * self.w(p + "layer_scalar")
        x = _norm(x, self.w("norm.weight"), self.eps)
        head = self.t.get("lm_head.weight", emb)
        logits = x @ head.T
        cap = c.get("final_logit_softcapping")
        return cap * torch.tanh(logits / cap) if cap else logits
