"""Plain-PyTorch fp32 forward of the supported decoder families: the numerics oracle.

This is the framework's equivalent of the reference's cpu-ref backend and
cacheless ``Model.Forward`` (internal/compute/cpuref.go:38-290,
internal/model/forward.go:45-434): every CUDA kernel and every engine path
is tested against it.  Semantics kept identical to the reference:

* RMSNorm ``x * rsqrt(mean(x^2) + eps) * w`` (cuda_kernels.cu:529-548).
* HF rotate_half RoPE with the angle computed in float64 (cuda_kernels.cu:551-567).
* SiLU-gated FFN; qkv bias (Qwen2); per-head q/k RMSNorm before RoPE (Qwen3); GELU-tanh gated FFN,
  score and logit soft-capping, sandwich norms, embedding scale (Gemma-2).
* MoE router: softmax over all experts, then top-k, renormalised when
  ``norm_topk_prob`` (internal/model/moe.go:279-311).
* Causal attention with GQA head groups.
* Qwen3.5 hybrid blocks: Gated DeltaNet token mixing on the linear layers (causal depthwise conv
  + SiLU, L2-normalised q/k, per-head decay exp(g) and write strength beta, the delta-rule state
  update S <- exp(g) S + k (beta (v - S^T k))^T, gated RMSNorm of the read-out), sigmoid output
  gate and partial rotary on the full-attention layers (internal/model/qwen35.go:32-561).
* gpt-oss blocks: a per-head sink logit that joins every softmax and is then dropped
  (internal/model/arch.go:304-333, softmaxDropSinkInPlace), output-projection bias, a biased
  top-k-then-softmax router, biased experts and the clamped OAI gate (internal/model/config.go:205-214).
"""
from __future__ import annotations

import math

import numpy as np
import torch

from ..config import ModelConfig


def softcap(x: torch.Tensor, cap: float) -> torch.Tensor:
    return cap * torch.tanh(x / cap) if cap > 0 else x


def act_fn(name: str, g: torch.Tensor) -> torch.Tensor:
    if name == "silu":
        return torch.nn.functional.silu(g)
    if name == "gelu_tanh":
        return torch.nn.functional.gelu(g, approximate="tanh")
    raise ValueError(f"unknown activation {name!r}")


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    inv = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return xf * inv * w.float()


def rope_cos_sin(positions: torch.Tensor, head_dim: int, theta: float, scaling=None, max_context: int | None = None
                 ) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin tables [T, head_dim/2] with angles evaluated in float64 (scaled RoPE variants included)."""
    from .rope import cos_sin
    c, s = cos_sin(positions, head_dim, theta, scaling, max_context)
    return c.to(positions.device), s.to(positions.device)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [T, H, D]; rotate_half pairs (j, j + D/2)."""
    half = x.shape[-1] // 2
    x0, x1 = x[..., :half], x[..., half:]
    c, s = cos[:, None, :], sin[:, None, :]
    return torch.cat([x0 * c - x1 * s, x1 * c + x0 * s], dim=-1)


def l2norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    return x * torch.rsqrt((x * x).sum(-1, keepdim=True) + eps)


def gated_delta_rule(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor, beta: torch.Tensor,
                     S: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Token-serial gated delta rule.  q, k [T, H, dk] (q already scaled), v [T, H, dv], g, beta
    [T, H], S [H, dk, dv] the state before the first token.  Returns (out [T, H, dv], final S)."""
    out = torch.empty(q.shape[0], q.shape[1], v.shape[-1], dtype=torch.float32, device=q.device)
    for t in range(q.shape[0]):
        S = S * torch.exp(g[t])[:, None, None]
        mem = torch.einsum("hkv,hk->hv", S, k[t])
        delta = (v[t] - mem) * beta[t][:, None]
        S = S + k[t][:, :, None] * delta[:, None, :]
        out[t] = torch.einsum("hkv,hk->hv", S, q[t])
    return out, S


def oai_gate(g: torch.Tensor, u: torch.Tensor, alpha: float, limit: float) -> torch.Tensor:
    """gpt-oss gated activation: (u + 1) * g * sigmoid(alpha * g), the gate clamped to <= limit and
    the linear branch to [-limit, limit] (limit 0: no clamp)."""
    if limit > 0:
        g = g.clamp(max=limit)
        u = u.clamp(-limit, limit)
    return (u + 1.0) * g * torch.sigmoid(alpha * g)


def moe_route(logits: torch.Tensor, k: int, norm_topk: bool, kind: str = "softmax_topk"
              ) -> tuple[torch.Tensor, torch.Tensor]:
    """Returns (weights [T,k], expert ids [T,k]).  "softmax_topk": softmax over every expert, then
    the top k (renormalised when ``norm_topk``); "topk_softmax": the top k logits, then a softmax
    over those k."""
    if kind == "topk_softmax":
        v, idx = torch.topk(logits.float(), k, dim=-1)
        return torch.softmax(v, dim=-1), idx
    p = torch.softmax(logits.float(), dim=-1)
    w, idx = torch.topk(p, k, dim=-1)
    if norm_topk:
        w = w / w.sum(-1, keepdim=True)
    return w, idx


class ReferenceModel:
    """fp32 forward over canonical GGUF-named tensors (already dequantized, HF row order)."""

    def __init__(self, cfg: ModelConfig, tensors: dict[str, torch.Tensor], device: str | torch.device = "cpu"):
        cfg.validate()
        self.cfg = cfg
        self.device = torch.device(device)
        self.t = {k: v.to(self.device, torch.float32) for k, v in tensors.items()}
        self.lora = None   # models.lora.LoRASet applied dynamically after each patched projection
        self.taps: dict[int, torch.Tensor] | None = None   # hidden tap: residual stream after layer i
        self.attn_observer = None   # callable(layer, probs [H, Tq, Tctx]) for every attention

    def set_lora(self, lora_set) -> None:
        self.lora = lora_set

    def mm(self, x: torch.Tensor, name: str) -> torch.Tensor:
        """x @ W^T (+ the active LoRA deltas of W)."""
        y = x @ self.t[name].T
        if self.lora is not None:
            d = self.lora.delta(name, x)
            if d is not None:
                y = y + d
        return y

    @classmethod
    def from_gguf(cls, path_or_file, device: str | torch.device = "cpu") -> "ReferenceModel":
        from .loader import load_reference_tensors
        cfg, tensors = load_reference_tensors(path_or_file)
        return cls(cfg, tensors, device)

    def w(self, name: str) -> torch.Tensor:
        return self.t[name]

    def embed(self, ids: torch.Tensor) -> torch.Tensor:
        e = self.t["token_embd.weight"][ids.to(self.device)]
        return e * self.cfg.embed_scale if self.cfg.embed_scale != 1.0 else e

    def lm_head(self, h: torch.Tensor) -> torch.Tensor:
        W = self.t["token_embd.weight"] if self.cfg.tie_embeddings else self.t["output.weight"]
        return softcap(h @ W.T, self.cfg.final_softcap)

    def _ffn(self, i: int, x: torch.Tensor) -> torch.Tensor:
        cfg, p = self.cfg, f"blk.{i}."
        if not cfg.is_moe:
            g = self.mm(x, p + "ffn_gate.weight")
            u = self.mm(x, p + "ffn_up.weight")
            return self.mm(act_fn(cfg.act, g) * u, p + "ffn_down.weight")
        logits = x @ self.w(p + "ffn_gate_inp.weight").T
        if cfg.moe_bias:
            logits = logits + self.w(p + "ffn_gate_inp.bias")
        wts, idx = moe_route(logits, cfg.n_experts_used, cfg.norm_topk_prob, cfg.router)
        G, U, D = self.w(p + "ffn_gate_exps.weight"), self.w(p + "ffn_up_exps.weight"), self.w(p + "ffn_down_exps.weight")
        if cfg.moe_bias:
            bg, bu, bd = (self.w(p + n) for n in ("ffn_gate_exps.bias", "ffn_up_exps.bias", "ffn_down_exps.bias"))
        out = torch.zeros_like(x)
        for t in range(x.shape[0]):
            for j in range(cfg.n_experts_used):
                e = int(idx[t, j])
                g, u = G[e] @ x[t], U[e] @ x[t]
                if cfg.moe_bias:
                    g, u = g + bg[e], u + bu[e]
                h = oai_gate(g, u, cfg.swiglu_alpha, cfg.swiglu_limit) if cfg.swiglu_alpha > 0 \
                    else act_fn(cfg.act, g) * u
                y = D[e] @ h
                if cfg.moe_bias:
                    y = y + bd[e]
                out[t] += wts[t, j] * y
        return out

    def _gdn(self, i: int, h: torch.Tensor, state) -> tuple[torch.Tensor, tuple]:
        """Gated DeltaNet token mixing of layer i over h [T, d].  ``state`` = (the last gdn_conv - 1
        conv inputs [gdn_conv - 1, C], the delta-rule state [v heads, dk, dv]) or None at position 0."""
        cfg, p = self.cfg, f"blk.{i}."
        T = h.shape[0]
        Hk, Hv, dk, dv, Kc = cfg.gdn_k_heads, cfg.gdn_v_heads, cfg.gdn_k_dim, cfg.gdn_v_dim, cfg.gdn_conv
        mixed = self.mm(h, p + "ssm_in_qkv.weight")                    # [T, C]
        C = mixed.shape[1]
        if state is None:
            state = (torch.zeros(Kc - 1, C, device=h.device), torch.zeros(Hv, dk, dv, device=h.device))
        xin = torch.cat([state[0], mixed])                               # [Kc - 1 + T, C]
        w = self.w(p + "ssm_conv1d.weight")                              # [C, Kc]
        conv = sum(xin[k:k + T] * w[:, k] for k in range(Kc))
        mixed = torch.nn.functional.silu(conv)
        q, k, v = torch.split(mixed, [Hk * dk, Hk * dk, Hv * dv], dim=-1)
        q, k, v = q.reshape(T, Hk, dk), k.reshape(T, Hk, dk), v.reshape(T, Hv, dv)
        if Hv > Hk:
            q, k = q.repeat_interleave(Hv // Hk, dim=1), k.repeat_interleave(Hv // Hk, dim=1)
        q, k = l2norm(q) * dk ** -0.5, l2norm(k)
        beta = torch.sigmoid(self.mm(h, p + "ssm_in_b.weight"))
        g = -torch.exp(self.w(p + "ssm_a")) * torch.nn.functional.softplus(
            self.mm(h, p + "ssm_in_a.weight") + self.w(p + "ssm_dt.bias"))
        o, S = gated_delta_rule(q, k, v, g, beta, state[1])
        z = self.mm(h, p + "ssm_in_z.weight").view(T, Hv, dv)
        o = rmsnorm(o, self.w(p + "ssm_norm.weight"), cfg.rms_eps) * torch.nn.functional.silu(z)
        return self.mm(o.reshape(T, Hv * dv), p + "ssm_out.weight"), (xin[-(Kc - 1):], S)

    def forward(self, ids: torch.Tensor, start_pos: int = 0,
                kv: list[tuple[torch.Tensor, torch.Tensor]] | None = None,
                hidden_only: bool = False) -> torch.Tensor:
        """Run T tokens at absolute positions start_pos.. ; ``kv`` (per layer [Tctx,Hkv,D]) is extended in place."""
        cfg = self.cfg
        ids = torch.as_tensor(ids, dtype=torch.long, device=self.device).reshape(-1)
        x = self.forward_band(self.embed(ids), start_pos, 0, cfg.n_layers, kv)
        x = rmsnorm(x, self.t["output_norm.weight"], cfg.rms_eps)
        return x if hidden_only else self.lm_head(x)

    def forward_band(self, x: torch.Tensor, start_pos: int, l0: int, l1: int,
                     kv: list[tuple[torch.Tensor, torch.Tensor]] | None = None) -> torch.Tensor:
        """Layers [l0, l1) on the residual stream x [T, d] (a pipeline stage's band).  ``kv`` holds
        the band's layers, index i - l0."""
        cfg = self.cfg
        T = x.shape[0]
        pos = torch.arange(start_pos, start_pos + T, device=self.device)
        cos, sin = rope_cos_sin(pos, cfg.rope_dim, cfg.rope_theta, cfg.rope_scaling, cfg.max_context)
        H, Hk, D, rd = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.rope_dim

        def rope(t):
            return apply_rope(t, cos, sin) if rd == D else torch.cat([apply_rope(t[..., :rd], cos, sin), t[..., rd:]], -1)

        for i in range(l0, l1):
            p = f"blk.{i}."
            h = rmsnorm(x, self.w(p + "attn_norm.weight"), cfg.rms_eps)
            if cfg.is_linear(i):
                j = i - l0
                state = kv[j] if kv is not None and len(kv) > j else None
                o, state = self._gdn(i, h, state)
                if kv is not None:
                    if len(kv) <= j:
                        kv.append(state)
                    else:
                        kv[j] = state
                x = x + o
                x = x + self._ffn(i, rmsnorm(x, self.w(p + "ffn_norm.weight"), cfg.rms_eps))
                if self.taps is not None:
                    self.taps[i] = x.detach().clone()
                continue
            q = self.mm(h, p + "attn_q.weight")
            gate = None
            if cfg.attn_out_gate:   # per head: D query dims, then D gate dims
                qg = q.view(T, H, 2 * D)
                q, gate = qg[..., :D].reshape(T, H * D), qg[..., D:].reshape(T, H * D)
            k = self.mm(h, p + "attn_k.weight")
            v = self.mm(h, p + "attn_v.weight")
            if cfg.qkv_bias:
                q = q + self.w(p + "attn_q.bias")
                k = k + self.w(p + "attn_k.bias")
                v = v + self.w(p + "attn_v.bias")
            q = q.view(T, H, D)
            k = k.view(T, Hk, D)
            v = v.view(T, Hk, D)
            if cfg.qk_norm:
                q = rmsnorm(q, self.w(p + "attn_q_norm.weight"), cfg.rms_eps)
                k = rmsnorm(k, self.w(p + "attn_k_norm.weight"), cfg.rms_eps)
            q = rope(q)
            k = rope(k)
            j = i - l0
            if kv is not None:
                if len(kv) <= j:
                    kv.append((k, v))
                else:
                    kv[j] = (torch.cat([kv[j][0], k]), torch.cat([kv[j][1], v]))
                K, V = kv[j]
            else:
                K, V = k, v
            a = attention(q, K, V, start_pos, cfg.layer_window(i),
                          None if self.attn_observer is None else (lambda pr, i=i: self.attn_observer(i, pr)),
                          scale=cfg.attn_scale, softcap_=cfg.attn_softcap,
                          sinks=self.w(p + "attn_sinks.weight") if cfg.attn_sinks else None)
            a = a.reshape(T, H * D)
            if gate is not None:
                a = a * torch.sigmoid(gate)
            o = self.mm(a, p + "attn_output.weight")
            if cfg.attn_out_bias:
                o = o + self.w(p + "attn_output.bias")
            if cfg.sandwich_norms:
                o = rmsnorm(o, self.w(p + "post_attention_norm.weight"), cfg.rms_eps)
            x = x + o
            h = rmsnorm(x, self.w(p + "ffn_norm.weight"), cfg.rms_eps)
            f = self._ffn(i, h)
            if cfg.sandwich_norms:
                f = rmsnorm(f, self.w(p + "post_ffw_norm.weight"), cfg.rms_eps)
            x = x + f
            if self.taps is not None:
                self.taps[i] = x.detach().clone()
        return x

    @torch.no_grad()
    def logit_lens(self, ids, layers: list[int] | None = None, top: int = 1) -> dict[int, torch.Tensor]:
        """Top-``top`` token ids of the final norm + LM head applied to the residual stream after
        each layer (the logit lens), for every position: {layer: [T, top]}."""
        self.taps = {}
        try:
            self.forward(torch.as_tensor(ids), hidden_only=True)
            taps = self.taps
        finally:
            self.taps = None
        out = {}
        for i in (layers if layers is not None else sorted(taps)):
            h = rmsnorm(taps[i], self.t["output_norm.weight"], self.cfg.rms_eps)
            out[i] = torch.topk(self.lm_head(h), top, dim=-1).indices
        return out

    @torch.no_grad()
    def generate_greedy(self, prompt: list[int], n_new: int) -> list[int]:
        kv: list = []
        logits = self.forward(torch.tensor(prompt), 0, kv)
        out = []
        nxt = int(torch.argmax(logits[-1]))
        pos = len(prompt)
        for _ in range(n_new):
            out.append(nxt)
            logits = self.forward(torch.tensor([nxt]), pos, kv)
            pos += 1
            nxt = int(torch.argmax(logits[-1]))
        return out


def attention(q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, start_pos: int, window: int = 0,
              observe=None, scale: float = 0.0, softcap_: float = 0.0,
              sinks: torch.Tensor | None = None) -> torch.Tensor:
    """q [T,H,D] at positions start_pos..; K,V [Tctx,Hk,D] covering positions 0..Tctx-1 (causal;
    window > 0: each query sees keys (qpos - window, qpos]).  sinks [H]: one extra logit per head
    that joins the softmax's normaliser and attends to nothing."""
    T, H, D = q.shape
    Tc, Hk, _ = K.shape
    g = H // Hk
    Kx = K.repeat_interleave(g, dim=1)
    Vx = V.repeat_interleave(g, dim=1)
    s = torch.einsum("thd,chd->htc", q.float(), Kx.float()) * (scale if scale > 0 else 1.0 / math.sqrt(D))
    s = softcap(s, softcap_)
    qpos = torch.arange(start_pos, start_pos + T, device=q.device)[:, None]
    kpos = torch.arange(Tc, device=q.device)[None, :]
    masked = kpos > qpos
    if window > 0:
        masked = masked | (kpos <= qpos - window)
    s = s.masked_fill(masked[None], float("-inf"))
    if sinks is not None:
        sk = sinks.float().to(s.device)[:, None, None].expand(H, T, 1)
        pr = torch.softmax(torch.cat([s, sk], dim=-1), dim=-1)[..., :-1]
    else:
        pr = torch.softmax(s, dim=-1)
    if observe is not None:
        observe(pr)
    return torch.einsum("htc,chd->thd", pr, Vx.float())


def numpy_seeded_ids(n: int, vocab: int, seed: int) -> list[int]:
    """Seeded uniform token ids (the benchmarks' synthetic prompts)."""
    rng = np.random.default_rng(seed)
    return rng.integers(0, vocab, size=n).tolist()
