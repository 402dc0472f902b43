"""DeepSeek-style sparse attention (the GLM-MoE-DSA attention): indexer scores, top-k selection and
attention over the selected keys, as device ops and as the plain PyTorch definitions they are
tested against.

A decode step of a DSA layer: the indexer projects the query into ``nh`` index heads ``iq`` and
keeps one index key ``ik[k]`` per cached position; ``score[k] = sum_h w[h] relu(scale <iq[h],
ik[k]>)`` over positions k <= qpos; the ``topk`` best positions (lower position first on ties) are
the only keys the attention heads see; attention uses MLA widths (query/key width ``kd`` differs
from the value width ``vd``).

Reference: glmDsaAttendCached / dsa_index (internal/model/glm_dsa.go, dsa_index.go) and the
device kernels of internal/compute/cuda_kernels.cu:773-907.
"""
from __future__ import annotations

import math

import torch


def index_scores_ref(iq: torch.Tensor, ik: torch.Tensor, w: torch.Tensor, qpos: int, scale: float) -> torch.Tensor:
    s = torch.relu((ik.double() @ iq.double().T) * scale) @ w.double()      # [n_keys]
    s[qpos + 1:] = -math.inf
    return s


def topk_ref(score: torch.Tensor, qpos: int, topk: int) -> list[int]:
    n = min(qpos + 1, score.numel())
    order = sorted(range(n), key=lambda i: (-float(score[i]), i))
    return order[:topk]


def sparse_attend_ref(q: torch.Tensor, kc: torch.Tensor, vc: torch.Tensor, sel: list[int], scale: float) -> torch.Tensor:
    K = kc[sel].float()                               # [n_sel, H, kd]
    V = vc[sel].float()                               # [n_sel, H, vd]
    p = torch.softmax(torch.einsum("hd,nhd->hn", q.float(), K) * scale, dim=-1)
    return torch.einsum("hn,nhv->hv", p, V)


def dsa_decode(q, kc, vc, iq, ik, w, qpos: int, topk: int, index_scale: float, attn_scale: float):
    """One query through the device ops: (out [H, vd], selected positions)."""
    from ..ops._ext import ext
    C = ext()
    score = C.dsa_index_score(iq.contiguous(), ik.contiguous(), w.contiguous(), qpos, index_scale)
    sel, count = C.dsa_topk(score, qpos, topk)
    out = C.dsa_sparse_attend(q.contiguous(), kc.contiguous(), vc.contiguous(), sel, count, attn_scale)
    return out, sel[: int(count.item())]
