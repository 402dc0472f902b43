"""Tensor parallelism over NCCL: the collectives between the per-rank GEMVs/GEMMs (the baseline).

Sharding (models/weights.py):
* q/k/v: by heads.  With fewer KV heads than ranks a KV head is replicated and its query
  group split (Qwen2.5-7B at TP=8: 4 + 3 query heads per rank);
* attention: local heads only;
* o_proj: row-parallel (split along its input).  A rank holds the block-aligned column range around
  its heads (``weights.o_proj_columns``), multiplies its heads' outputs into a partial of the whole
  output row, and the partials are all-reduced into the replicated residual stream;
* gate/up: split by FFN rows in whole 256-wide super-blocks; down: split the same way along
  its input (K) dim -> partial sums -> all-reduce;
* lm_head: split by vocab rows -> all-gather of logits (or a distributed argmax, fused path).

Megatron's column/row scheme, the reference's TP (internal/model/tensor_parallel_forward.go:456-527)
on host f32 buffers with an AllReduceSum after o_proj and after down (:246, :371), cacheless prefill
only; this one runs decode and prefill on the GPU.

This class is the NCCL baseline: the product path (``parallel/p2p.py``, ``P2PTP``) moves both
all-reduces into the GEMV epilogue over peer memory.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import kernels as K


class _ActView:
    """ActQ-compatible view (codes ``q`` [B, K] int8, ``ds`` [B, K/32, 2] f32) over raw storage."""

    def __init__(self, q: torch.Tensor, ds: torch.Tensor, K: int):
        self.q, self.ds, self.K = q, ds, K


class NcclTP:
    def __init__(self, group, weights, max_batch: int, device):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        cfg = weights.cfg
        self.cfg = cfg
        self.D = cfg.head_dim
        self.o_cols = weights.o_cols
        self.Hq_local = len(weights.q_heads)
        B = max_batch
        self.tmp = torch.zeros(B, cfg.d_model, dtype=torch.float32, device=device)
        # every rank gathers ceil(V/T) logits (ranks with fewer real rows pad with -inf)
        self.Vl = -(-cfg.vocab_size // self.world)
        self.Vl_real = weights.lm_head.rows
        self.logits_local = torch.full((B, self.Vl), float("-inf"), dtype=torch.float32, device=device)
        self.logits_all = torch.zeros(self.world * B * self.Vl, dtype=torch.float32, device=device)
        self._act_view = None
        self._o_dense: dict[int, torch.Tensor] = {}

    # ---------------------------------------------------------------------------------
    def attn_out(self, rn) -> _ActView:
        """This rank's heads' columns inside the o_proj input slice (rows of a1 - a0 elements)."""
        if self._act_view is None:
            a0, a1, c0, _ = self.o_cols
            off = c0 - a0
            act = rn.act_attn
            self._act_view = _ActView(act.q.view(-1)[off:], act.ds.view(-1)[off // 16:], a1 - a0)
        return self._act_view

    def attention(self, rn, i: int, B: int, bt, ctx, n_split: int) -> None:
        """Decode attention of the local heads, written int8-quantized into the o_proj input slice."""
        kv = rn.kv
        # the split merge runs as its own kernel unless attention_merge is on, as on one GPU (merging in
        # the last split's CTA serialises a long tail: 0.7 ms/step slower on Qwen2.5-7B at batch 5)
        K.decode_attention(rn.q[:B], kv.k[i], kv.v[i], bt, ctx, n_split, pages_per_split=max(1, rn.dec_pps),
                           act=self.attn_out(rn), workspace=rn.attn_ws,
                           tickets=rn.attn_tickets if rn.attn_merge else None, ldo=self.o_cols[1] - self.o_cols[0],
                           window=rn.cfg.layer_window(i), **rn.cascade_args(B, rn.cfg.layer_window(i)))

    def decode_attn_o(self, rn, i: int, B: int, bt, ctx, n_split: int) -> None:
        self.attention(rn, i, B, bt, ctx, n_split)
        t = self.tmp[:B]
        K.gemv(rn.w.layers[i].o, rn.act_attn, B, t, None, K.EPI_STORE)
        dist.all_reduce(t, group=self.group)
        rn.x[:B].add_(t)

    def decode_down(self, rn, i: int, B: int) -> None:
        t = self.tmp[:B]
        K.gemv(rn.w.layers[i].down, rn.ffn_in, B, t, None, K.EPI_STORE)
        dist.all_reduce(t, group=self.group)
        rn.x[:B].add_(t)

    def _gather_logits(self, B: int, out: torch.Tensor) -> None:
        la = self.logits_all[:self.world * B * self.Vl]
        dist.all_gather_into_tensor(la, self.logits_local[:B].reshape(-1), group=self.group)
        V = out.shape[1]
        full = la.view(self.world, B, self.Vl).permute(1, 0, 2).reshape(B, -1)
        out[:B].copy_(full[:, :V])

    def lm_head(self, rn, B: int) -> None:
        K.gemv(rn.w.lm_head, rn.lm_in, B, self.logits_local[:B, :self.Vl_real], None, K.EPI_STORE)
        self._gather_logits(B, rn.logits)

    def lm_head_to(self, rn, n: int, out: torch.Tensor) -> None:
        K.gemv(rn.w.lm_head, rn.lm_in, n, self.logits_local[:n, :self.Vl_real], None, K.EPI_STORE)
        self._gather_logits(n, out)

    # ---------------------------------------------------------------------------------
    def o_dense_local(self, rn, i: int) -> torch.Tensor:
        """bf16 [d, n_local_heads * D]: the columns of o_proj that this rank's heads feed (prefill)."""
        w = self._o_dense.get(i)
        if w is None:
            a0, _, c0, c1 = self.o_cols
            w = rn.w.layers[i].o.dense()[:, c0 - a0:c1 - a0].contiguous()
            self._o_dense[i] = w
        return w

    def prefill_attn_o(self, rn, i: int, ab: torch.Tensor, x: torch.Tensor) -> None:
        part = torch.empty_like(x)
        K.gemm(ab, self.o_dense_local(rn, i), part, K.EPI_STORE)
        dist.all_reduce(part, group=self.group)
        x.add_(part)

    def prefill_down(self, rn, i: int, hb2: torch.Tensor, x: torch.Tensor) -> None:
        t = torch.empty_like(x)
        K.gemm(hb2, rn.w.layers[i].down, t, K.EPI_STORE)
        dist.all_reduce(t, group=self.group)
        x.add_(t)

    # ---------------------------------------------------------------------------------
    def reduce_partial(self, rn, i: int, B: int, fill) -> None:
        """x += all-reduce(partial), where fill(partial) writes this rank's contribution."""
        t = self.tmp[:B]
        fill(t)
        dist.all_reduce(t, group=self.group)
        rn.x[:B].add_(t)

    def prefill_reduce(self, part: torch.Tensor, x: torch.Tensor) -> None:
        dist.all_reduce(part, group=self.group)
        x.add_(part)
