"""MiniMax-M3 sparse attention (MSA): block-granular key selection over the real GQA K/V.

For every query a lightning indexer scores every cached key; the scores of the causal keys
(position <= the query's) are max-pooled into blocks of ``block`` consecutive positions (block id =
position // block; a block counts when it holds at least one causal key with a finite score).  The
query then attends to the union of

* the ``topk`` blocks with the highest pooled score (equal scores: the lower block id first), and
* the ``local`` most recent candidate blocks (the query's own block and those just behind it),

and the per-block choice is broadcast onto every causal key of the chosen blocks; softmax attention
runs over the admitted keys only.  Where DSA (``models/dsa.py``) picks individual keys, MSA picks
whole blocks with an always-on local window; the sparse softmax after the choice is the same.

Everything here is batched over queries as dense masks (``[Tq, n_blocks]``, ``[Tq, Tk]``) so it runs
as a handful of tensor ops on either device.  Like the reference, this covers the selection and the
sparse attention; the learned indexer projections of a real checkpoint are not wired into a model.

Two selection rules exist: ``select_blocks`` is the union above; ``select_blocks_fixed`` is the
fixed-count rule of the MiniMax-M3 forward (local blocks forced in, displacing the lowest-scored
ones), with the block scores max-pooled over the indexer's heads (``pooled_over_heads``).

Reference: internal/model/msa_index.go (msaBlockScores :37-68, msaSelectBlocks :70-118,
msaSelectedKeyPositions :120-160, msaAttention :162-192); internal/model/minimax_m3.go
(minimaxIndexerSelectBlocks :223-263, minimaxSelectBlocks :265-298).
"""
from __future__ import annotations

import math

import torch


def block_scores(scores: torch.Tensor, key_pos: torch.Tensor, q_pos: torch.Tensor, block: int
                 ) -> torch.Tensor:
    """scores [Tq, Tk] (the indexer's per-key scores), key_pos [Tk], q_pos [Tq] -> pooled [Tq, nb]
    (-inf where a block holds no causal key with a finite score; NaN scores are skipped)."""
    if block <= 0:
        raise ValueError("block size must be positive")
    if (key_pos < 0).any() or (q_pos < 0).any():
        raise ValueError("positions must be non-negative")
    if torch.unique(key_pos).numel() != key_pos.numel():
        raise ValueError("duplicate key positions in the cache layout")
    s = scores.double().clone()
    causal = key_pos[None, :] <= q_pos[:, None]
    s[~causal | torch.isnan(s)] = -math.inf
    nb = int(key_pos.max()) // block + 1 if key_pos.numel() else 0
    bid = (key_pos // block).expand_as(s)
    out = torch.full((s.shape[0], nb), -math.inf, dtype=torch.float64, device=s.device)
    return out.scatter_reduce(1, bid, s, reduce="amax", include_self=True)


def select_blocks(pooled: torch.Tensor, topk: int, local: int) -> torch.Tensor:
    """pooled [Tq, nb] -> bool [Tq, nb]: per query the top-``topk`` candidate blocks by pooled score
    (ties: lower id) united with the ``local`` highest-id candidate blocks."""
    if topk < 0 or local < 0:
        raise ValueError("topk and local must be non-negative")
    cand = pooled > -math.inf
    nb = pooled.shape[1]
    # rank of each candidate among the query's candidates counted from the newest (0 = newest)
    from_newest = cand.flip(1).cumsum(1).flip(1) - 1
    sel = cand & (from_newest < local)
    if topk > 0 and nb > 0:
        # sort by (-score, id): a stable sort on -score over ids ascending keeps lower ids first on ties
        key = torch.where(cand, -pooled, torch.full_like(pooled, math.inf))
        order = torch.sort(key, dim=1, stable=True).indices[:, :topk]
        top = torch.zeros_like(cand)
        top.scatter_(1, order, True)
        sel |= top & cand
    return sel


def select_blocks_fixed(pooled: torch.Tensor, q_pos: torch.Tensor, block: int, topk: int, local: int
                        ) -> torch.Tensor:
    """The fixed-count selection of the MiniMax-M3 forward: the ``local`` blocks ending at the
    query's own block are forced to +inf, then exactly min(topk, candidates) blocks are kept by
    score (ties: lower id), so a forced local block displaces the lowest-scored one instead of
    adding to the set.  pooled [Tq, nb] -> bool [Tq, nb]."""
    if topk < 0 or local < 0:
        raise ValueError("topk and local must be non-negative")
    cand = pooled > -math.inf
    nb = pooled.shape[1]
    ids = torch.arange(nb, device=pooled.device)[None, :]
    qb = (q_pos // block)[:, None]
    forced = cand & (ids <= qb) & (ids > qb - local)
    key = torch.where(forced, torch.full_like(pooled, -math.inf), -pooled)
    key = torch.where(cand, key, torch.full_like(pooled, math.inf))
    order = torch.sort(key, dim=1, stable=True).indices
    n = cand.sum(1).clamp(max=topk)
    rank = torch.empty_like(order)
    rank.scatter_(1, order, torch.arange(nb, device=pooled.device).expand_as(order))
    return cand & (rank < n[:, None])


def pooled_over_heads(scores: torch.Tensor, key_pos: torch.Tensor, q_pos: torch.Tensor, block: int) -> torch.Tensor:
    """Block scores of a multi-head indexer: per-head scores [Tq, heads, Tk] max-pooled over each
    block and then over the heads -> [Tq, nb] (one selection shared by every attention head)."""
    per = [block_scores(scores[:, h], key_pos, q_pos, block) for h in range(scores.shape[1])]
    return torch.stack(per, 0).amax(0)


def key_mask(sel: torch.Tensor, key_pos: torch.Tensor, q_pos: torch.Tensor, block: int) -> torch.Tensor:
    """Block choice [Tq, nb] -> admitted keys bool [Tq, Tk] (causal keys of chosen blocks)."""
    bid = key_pos // block
    return sel[:, bid] & (key_pos[None, :] <= q_pos[:, None])


def msa_attention(q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, scores: torch.Tensor, q_pos: torch.Tensor,
                  key_pos: torch.Tensor, block: int, topk: int, local: int, scale: float = 0.0
                  ) -> tuple[torch.Tensor, torch.Tensor]:
    """q [Tq, H, D], K / V [Tk, Hk, D] (GQA), scores [Tq, Tk] -> (out [Tq, H, D] fp32, admitted
    keys [Tq, Tk]).  A query that admits no key raises (with ``local`` or ``topk`` >= 1 that only
    happens when it sees no causal key with a finite score)."""
    mask = key_mask(select_blocks(block_scores(scores, key_pos, q_pos, block), topk, local), key_pos, q_pos, block)
    if not bool(mask.any(1).all()):
        raise ValueError("a query admitted no key")
    H, Hk, D = q.shape[1], K.shape[1], q.shape[2]
    g = H // Hk
    Kx, Vx = K.float().repeat_interleave(g, dim=1), V.float().repeat_interleave(g, dim=1)
    s = torch.einsum("thd,khd->htk", q.float(), Kx) * (scale if scale > 0 else 1.0 / math.sqrt(D))
    s = s.masked_fill(~mask[None], -math.inf)
    return torch.einsum("htk,khd->thd", torch.softmax(s, dim=-1), Vx), mask
