"""Tensor parallelism over NCCL: the collectives between the per-rank GEMVs/GEMMs.

Sharding (models/weights.py):
* q/k/v: by heads.  With fewer KV heads than ranks a KV head is replicated and its query
  group split (Qwen2.5-7B at TP=8: 4 + 3 query heads per rank);
* attention: local heads only;
* o_proj: whole on every rank.  The attention outputs of all heads are all-gathered (int8
  codes + per-32 scales for decode, bf16 for prefill) and every rank applies the full
  projection, so the residual stream stays replicated with a single collective;
* gate/up: split by FFN rows in whole 256-wide super-blocks; down: split the same way along
  its input (K) dim -> partial sums -> all-reduce;
* lm_head: split by vocab rows -> all-gather of logits.

The reference's TP (internal/model/tensor_parallel_forward.go:456-527) is the Megatron
column/row scheme on host f32 buffers with an AllReduceSum after o_proj and down
(:246, :371), cacheless prefill only; this one runs decode and prefill on the GPU.

This class is the NCCL baseline.  The fused path (parallel/fused.py) replaces the
collectives with in-kernel peer-memory transfers.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import kernels as K


class NcclTP:
    def __init__(self, group, weights, max_batch: int, device):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        cfg = weights.cfg
        self.cfg = cfg
        D = cfg.head_dim
        self.D = D
        # head ownership of every rank (deterministic: recomputed, not communicated)
        from ..models.weights import head_assignment
        owners = [head_assignment(cfg, r, self.world)[0] for r in range(self.world)]
        self.maxHq = max(len(o) for o in owners)
        slot = [0] * cfg.n_heads
        for r, heads in enumerate(owners):
            for j, h in enumerate(heads):
                slot[h] = r * self.maxHq + j
        self.head_slot = torch.tensor(slot, dtype=torch.long, device=device)
        self.Hq_local = len(owners[self.rank])
        B = max_batch
        self.act_local = K.ActQ(B, self.maxHq * D, device)
        # gather targets are flat: [world, b, ...] views of their first world*b rows stay contiguous
        self.recv_q = torch.zeros(self.world * B * self.maxHq * D, dtype=torch.int8, device=device)
        self.recv_ds = torch.zeros(self.world * B * self.maxHq * D // 16, dtype=torch.float32, device=device)
        self.tmp = torch.zeros(B, cfg.d_model, dtype=torch.float32, device=device)
        # every rank gathers ceil(V/T) logits (ranks with fewer real rows pad with -inf)
        self.Vl = -(-cfg.vocab_size // self.world)
        self.Vl_real = weights.lm_head.rows
        self.logits_local = torch.full((B, self.Vl), float("-inf"), dtype=torch.float32, device=device)
        self.logits_all = torch.zeros(self.world * B * self.Vl, dtype=torch.float32, device=device)

    # ---------------------------------------------------------------------------------
    def _gather_heads_q(self, B: int, act_dst) -> None:
        D, H, Wd = self.D, self.cfg.n_heads, self.world
        rq = self.recv_q[:Wd * B * self.maxHq * D]
        rd = self.recv_ds[:Wd * B * self.maxHq * D // 16]
        dist.all_gather_into_tensor(rq, self.act_local.q[:B].reshape(-1), group=self.group)
        dist.all_gather_into_tensor(rd, self.act_local.ds[:B].reshape(-1), group=self.group)
        q = rq.view(Wd, B, self.maxHq, D).permute(1, 0, 2, 3).reshape(B, -1, D)
        ds = rd.view(Wd, B, self.maxHq, D // 32, 2).permute(1, 0, 2, 3, 4)
        ds = ds.reshape(B, -1, D // 32, 2)
        act_dst.q[:B].view(B, H, D).copy_(q.index_select(1, self.head_slot))
        act_dst.ds[:B].view(B, H, D // 32, 2).copy_(ds.index_select(1, self.head_slot))

    def decode_attn_o(self, rn, i: int, B: int, bt, ctx, n_split: int) -> None:
        kv = rn.kv
        if self.Hq_local < self.maxHq:  # pad slots of ranks with fewer heads stay zero
            self.act_local.q[:B].zero_()
            self.act_local.ds[:B].zero_()
        K.decode_attention(rn.q[:B], kv.k[i], kv.v[i], bt, ctx, n_split, act=self.act_local, workspace=rn.attn_ws,
                           tickets=rn.attn_tickets, ldo=self.maxHq * self.D, window=rn.cfg.layer_window(i),
                           **rn.cascade_args(B, rn.cfg.layer_window(i)))
        self._gather_heads_q(B, rn.act_attn)
        K.gemv(rn.w.layers[i].o, rn.act_attn, B, rn.x[:B], None, K.EPI_ADD)

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
    def prefill_attn_o(self, rn, i: int, ab: torch.Tensor, x: torch.Tensor) -> None:
        T = ab.shape[0]
        D = self.D
        send = torch.zeros(T, self.maxHq * D, dtype=torch.bfloat16, device=ab.device)
        send[:, :ab.shape[1]].copy_(ab)
        recv = torch.empty(self.world, T, self.maxHq * D, dtype=torch.bfloat16, device=ab.device)
        dist.all_gather_into_tensor(recv.view(-1), send.view(-1), group=self.group)
        full = recv.view(self.world, T, self.maxHq, D).permute(1, 0, 2, 3).reshape(T, -1, D)
        full = full.index_select(1, self.head_slot).reshape(T, -1).contiguous()
        K.gemm(full, rn.w.layers[i].o, x, K.EPI_ADD)

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
