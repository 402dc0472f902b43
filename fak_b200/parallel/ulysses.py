"""Ulysses-style sequence parallelism for long single prompts: attention re-sharded by all-to-all.

Each of P ranks holds an equal, contiguous slice of the sequence (rank r: tokens
[r T/P, (r+1) T/P)) for every head.  Attention needs every key of a head, so before it one
all-to-all turns the sequence-sharded q / k / v [T/P, H, D] into head-sharded [T, H/P, D] (rank r
keeps heads [r H/P, (r+1) H/P) for the whole sequence); each rank runs ordinary causal attention
over its heads; a second all-to-all turns the result back into the sequence shard.  Per rank the
traffic is 3 inputs + 1 output of T/P x H x D each, independent of P, and the attention kernel
itself is unchanged.

Query and KV head counts must both divide by P (each rank owns whole GQA groups).  The transport
is ``torch.distributed.all_to_all_single`` (NCCL on GPUs, gloo on CPU).

The reference has no sequence or context parallelism (its long-context tools are window trim,
scaled RoPE, KV precision tiers and prefix reuse); this is an addition for prompts whose
attention does not fit one GPU's time budget.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist


def _world(group) -> int:
    return dist.get_world_size(group)


def seq_to_head(x: torch.Tensor, group=None) -> torch.Tensor:
    """[T/P, H, D] sequence shard -> [T, H/P, D] head shard (sequence in rank order)."""
    P = _world(group)
    Tl, H, D = x.shape
    if H % P:
        raise ValueError(f"{H} heads do not split over {P} ranks")
    send = x.reshape(Tl, P, H // P, D).permute(1, 0, 2, 3).contiguous()     # [P, T/P, H/P, D]
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    return recv.reshape(P * Tl, H // P, D)


def head_to_seq(y: torch.Tensor, group=None) -> torch.Tensor:
    """[T, H/P, D] head shard -> [T/P, H, D] sequence shard (inverse of ``seq_to_head``)."""
    P = _world(group)
    T, Hl, D = y.shape
    if T % P:
        raise ValueError(f"{T} tokens do not split over {P} ranks")
    send = y.reshape(P, T // P, Hl, D).contiguous()
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)                          # [P (head chunk), T/P, H/P, D]
    return recv.permute(1, 0, 2, 3).reshape(T // P, P * Hl, D)


def ulysses_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, group=None,
                      attn: Callable | None = None, **attn_kw) -> torch.Tensor:
    """Causal attention of a sequence-sharded prompt.  q [T/P, H, D], k / v [T/P, Hk, D] on every
    rank (positions from 0) -> this rank's output rows [T/P, H, D].  ``attn(q, K, V, 0, **attn_kw)``
    is the single-device attention (default: ``models.reference.attention``)."""
    P = _world(group)
    if k.shape[1] % P:
        raise ValueError(f"{k.shape[1]} KV heads do not split over {P} ranks")
    if attn is None:
        from ..models.reference import attention as attn
    qh, kh, vh = seq_to_head(q, group), seq_to_head(k, group), seq_to_head(v, group)
    out = attn(qh, kh, vh, 0, **attn_kw)
    return head_to_seq(out.to(q.dtype), group)
