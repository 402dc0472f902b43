"""GLM-MoE-DSA (GLM-5 family) on the fp32 reference path: multi-head latent attention (MLA) whose
keys are chosen per query by a DSA indexer, a sigmoid group-limited MoE router with shared
experts, and dense FFNs on the first layers.

Per layer (pre-norm residual blocks):

* MLA: q = W_qb RMSNorm(W_qa x), split per head into (nope, rope) parts; the latent
  c = W_kva x splits into (c_kv, k_rope); k_nope, v = W_kvb RMSNorm(c_kv) per head; the rope part
  of the key is one vector shared by every head.  RoPE (rotate-half pairs) on the rope parts only.
* DSA indexer: index queries W_iq RMSNorm(W_qa x) with ``index_n_heads`` heads and one index key
  LayerNorm(W_ik x) per position (RoPE on their FIRST ``qk_rope_head_dim`` dims); the score of key
  t for query s is sum_h w_h(s) relu(scale <iq_h(s), ik(t)>) with w = W_w x / sqrt(index heads);
  each query attends to its ``index_topk`` best-scored causal keys only (``models/dsa.py`` holds
  the same score / selection / sparse attention as device kernels).
* FFN: dense SwiGLU on "dense" layers; on "sparse" layers sigmoid router scores plus a correction
  bias pick ``topk_group`` groups by the sum of each group's two best scores, then the top-k
  experts inside them; the weights are the plain sigmoid scores, normalised when
  ``norm_topk_prob``, times ``routed_scaling_factor``; shared experts are always added.

The model reads a Hugging Face checkpoint (config.json + safetensors) under its own tensor names
and runs whole sequences (no cache), as the reference's cacheless GLM-DSA forward does.

Reference: internal/model/glm_dsa.go (MLA + DSA forward), dsa_index.go (indexer score, top-k),
internal/model/moe.go (sigmoid group-limited router with correction bias and shared experts).
"""
from __future__ import annotations

import glob
import json
import math
import os

import torch

from .hf import _to_f32, read_safetensors
from .reference import rmsnorm


def _rot(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """rotate-half RoPE over the last dim; cos / sin [T, dim/2] broadcast over the middle dims."""
    h = x.shape[-1] // 2
    x0, x1 = x[..., :h], x[..., h:]
    shape = (cos.shape[0],) + (1,) * (x.dim() - 2) + (h,)
    c, s = cos.view(shape), sin.view(shape)
    return torch.cat([x0 * c - x1 * s, x1 * c + x0 * s], dim=-1)


class GlmDsaReference:
    def __init__(self, hf: dict, tensors: dict[str, torch.Tensor]):
        self.c = hf
        self.t = {k: v.float() for k, v in tensors.items()}
        c = hf
        self.L = int(c["num_hidden_layers"])
        self.H = int(c["num_attention_heads"])
        self.nope, self.rope_d, self.vd = int(c["qk_nope_head_dim"]), int(c["qk_rope_head_dim"]), int(c["v_head_dim"])
        self.eps = float(c.get("rms_norm_eps", 1e-6))
        self.mlp_types = c.get("mlp_layer_types") or (
            ["dense"] * int(c.get("first_k_dense_replace", 0)) + ["sparse"] * (self.L - int(c.get("first_k_dense_replace", 0))))
        rp = c.get("rope_parameters") or {}
        self.theta = float(rp.get("rope_theta") or c.get("rope_theta") or 10000.0)

    @classmethod
    def from_hf(cls, model_dir: str) -> "GlmDsaReference":
        with open(os.path.join(model_dir, "config.json")) as f:
            hf = json.load(f)
        t = {}
        for p in sorted(glob.glob(os.path.join(model_dir, "*.safetensors"))):
            for n, (dt, shape, arr) in read_safetensors(p).items():
                t[n] = torch.from_numpy(_to_f32(dt, arr).reshape(shape).copy())
        return cls(hf, t)

    def w(self, n: str) -> torch.Tensor:
        return self.t[n]

    def _cos_sin(self, T: int) -> tuple[torch.Tensor, torch.Tensor]:
        d = self.rope_d
        inv = 1.0 / (self.theta ** (torch.arange(0, d, 2, dtype=torch.float64) / d))
        ang = torch.arange(T, dtype=torch.float64)[:, None] * inv[None, :]
        return torch.cos(ang).float(), torch.sin(ang).float()

    def index_topk(self, p: str, x: torch.Tensor, q_res: torch.Tensor, cos, sin) -> torch.Tensor:
        """Selected key positions [T, min(index_topk, T)] of every query (the DSA indexer)."""
        c = self.c
        nh, hd, rd = int(c["index_n_heads"]), int(c["index_head_dim"]), self.rope_d
        T = x.shape[0]
        q = (q_res @ self.w(p + "indexer.wq_b.weight").T).view(T, nh, hd)
        q = torch.cat([_rot(q[..., :rd], cos, sin), q[..., rd:]], -1)
        k = torch.nn.functional.layer_norm(x @ self.w(p + "indexer.wk.weight").T, (hd,),
                                           self.w(p + "indexer.k_norm.weight"), self.w(p + "indexer.k_norm.bias"), 1e-6)
        k = torch.cat([_rot(k[:, None, :rd], cos, sin)[:, 0], k[:, rd:]], -1)
        wts = (x @ self.w(p + "indexer.weights_proj.weight").T) * nh ** -0.5            # [T, nh]
        s = torch.relu(torch.einsum("shd,td->sht", q, k) * hd ** -0.5)
        score = torch.einsum("sht,sh->st", s, wts)
        causal = torch.ones(T, T, dtype=torch.bool).tril()
        score = score.masked_fill(~causal, -math.inf)
        return score.topk(min(int(c["index_topk"]), T), dim=-1).indices

    def attention(self, i: int, x: torch.Tensor, cos, sin) -> torch.Tensor:
        p = f"model.layers.{i}.self_attn."
        T, H, nope, rd, vd = x.shape[0], self.H, self.nope, self.rope_d, self.vd
        if p + "q_a_proj.weight" in self.t:
            q_res = rmsnorm(x @ self.w(p + "q_a_proj.weight").T, self.w(p + "q_a_layernorm.weight"), 1e-6)
            q = q_res @ self.w(p + "q_b_proj.weight").T
        else:
            raise ValueError("the DSA indexer reads the q_lora residual: checkpoints without q_a_proj are "
                             "not GLM-MoE-DSA")
        q = q.view(T, H, nope + rd)
        q = torch.cat([q[..., :nope], _rot(q[..., nope:], cos, sin)], -1)
        lat = x @ self.w(p + "kv_a_proj_with_mqa.weight").T
        ckv, k_rope = lat[:, :-rd], lat[:, -rd:]
        kv = (rmsnorm(ckv, self.w(p + "kv_a_layernorm.weight"), 1e-6) @ self.w(p + "kv_b_proj.weight").T).view(T, H, nope + vd)
        k_rope = _rot(k_rope[:, None, :], cos, sin).expand(T, H, rd)
        k = torch.cat([kv[..., :nope], k_rope], -1)
        v = kv[..., nope:]
        s = torch.einsum("shd,thd->hst", q, k) * (nope + rd) ** -0.5
        allowed = torch.zeros(T, T, dtype=torch.bool)
        allowed.scatter_(1, self.index_topk(p, x, q_res, cos, sin), True)
        allowed &= torch.ones(T, T, dtype=torch.bool).tril()
        s = s.masked_fill(~allowed[None], -math.inf)
        o = torch.einsum("hst,thd->shd", torch.softmax(s, -1), v).reshape(T, H * vd)
        return o @ self.w(p + "o_proj.weight").T

    def _mlp(self, p: str, x: torch.Tensor) -> torch.Tensor:
        g = x @ self.w(p + "gate_proj.weight").T
        u = x @ self.w(p + "up_proj.weight").T
        return (torch.nn.functional.silu(g) * u) @ self.w(p + "down_proj.weight").T

    def route(self, p: str, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """(expert ids [T, k], weights [T, k]) of the sigmoid group-limited router."""
        c = self.c
        E, k, G, kg = int(c["n_routed_experts"]), int(c["num_experts_per_tok"]), int(c["n_group"]), int(c["topk_group"])
        sc = torch.sigmoid(x @ self.w(p + "gate.weight").T)
        choice = sc + self.w(p + "gate.e_score_correction_bias")
        grp = choice.view(-1, G, E // G).topk(min(2, E // G), dim=-1).values.sum(-1)
        keep = torch.zeros_like(grp, dtype=torch.bool).scatter_(1, grp.topk(kg, dim=-1).indices, True)
        choice = choice.masked_fill(~keep.repeat_interleave(E // G, dim=1), 0.0)
        idx = choice.topk(k, dim=-1).indices
        wts = sc.gather(1, idx)
        if c.get("norm_topk_prob", True):
            wts = wts / (wts.sum(-1, keepdim=True) + 1e-20)
        return idx, wts * float(c.get("routed_scaling_factor", 1.0))

    def moe(self, i: int, x: torch.Tensor) -> torch.Tensor:
        p = f"model.layers.{i}.mlp."
        idx, wts = self.route(p, x)
        GU, D = self.w(p + "experts.gate_up_proj"), self.w(p + "experts.down_proj")
        I = D.shape[-1]
        out = torch.zeros_like(x)
        for t in range(x.shape[0]):
            for j in range(idx.shape[1]):
                e = int(idx[t, j])
                gu = GU[e] @ x[t]
                out[t] += wts[t, j] * (D[e] @ (torch.nn.functional.silu(gu[:I]) * gu[I:]))
        return out + self._mlp(p + "shared_experts.", x)

    @torch.no_grad()
    def forward(self, ids) -> torch.Tensor:
        ids = torch.as_tensor(ids, dtype=torch.long).reshape(-1)
        x = self.w("model.embed_tokens.weight")[ids]
        cos, sin = self._cos_sin(ids.numel())
        for i in range(self.L):
            p = f"model.layers.{i}."
            x = x + self.attention(i, rmsnorm(x, self.w(p + "input_layernorm.weight"), self.eps), cos, sin)
            h = rmsnorm(x, self.w(p + "post_attention_layernorm.weight"), self.eps)
            x = x + (self.moe(i, h) if self.mlp_types[i] == "sparse" else self._mlp(p + "mlp.", h))
        x = rmsnorm(x, self.w("model.norm.weight"), self.eps)
        head = self.t.get("lm_head.weight", self.w("model.embed_tokens.weight"))
        return x @ head.T
