"""Tensor-parallel decode with in-kernel peer-memory collectives (the fused path).

Every rank allocates one symmetric buffer (torch symmetric memory: same layout on every rank,
each rank's buffer mapped into every peer's address space over NVLink/NVSwitch) holding

* ``flags``  -- per-(site, CTA, source-rank) epoch flags of the cross-rank barriers;
* ``act``    -- the gathered int8 attention output (codes + per-32 (scale, sum)) of ALL heads;
* ``parts``  -- one fp32 [B, d] partial-sum slot per layer for the down-projection all-reduce;
* ``cand``   -- (value, id) argmax candidates for greedy sampling over the vocab shards.

Per decode layer the attention kernel writes its heads' quantized output straight into this
rank's ``act`` columns, one all-gather kernel pushes those columns into every peer's ``act``,
the o_proj GEMV reads the full ``act`` locally; the down-projection GEMV all-reduces in its own
epilogue: the warp that finishes a 16-row tile pushes the tile's partial to every rank, waits
for the other ranks' partials of that tile and adds their rank-order sum to the residual (one
kernel, the transfer of each tile overlapping the GEMV of the others).  Batches above 32 tokens
fall back to the GEMV + all-reduce kernel pair.
Greedy decoding ends with a distributed argmax instead of gathering 152k logits.  Prefill keeps
the NCCL collectives of ``NcclTP`` (large messages, bandwidth-bound).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import kernels as K
from ..ops._ext import ext
from .tp import NcclTP

MAX_CTAS = 64
MAX_W = 8
AR_CTAS = 16
AG_CTAS = 2


def _align(n: int, a: int = 256) -> int:
    return (n + a - 1) // a * a


class _ActView:
    """ActQ-compatible view (codes ``q`` [B, K] int8, ``ds`` [B, K/32, 2] f32) over raw storage."""

    def __init__(self, q: torch.Tensor, ds: torch.Tensor, K: int):
        self.q, self.ds, self.K = q, ds, K


class P2PTP(NcclTP):
    def __init__(self, group, weights, max_batch: int, device):
        super().__init__(group, weights, max_batch, device)
        import torch.distributed._symmetric_memory as symm_mem
        cfg = self.cfg
        if self.world > MAX_W:
            raise ValueError(f"P2P collectives support up to {MAX_W} ranks")
        B, H, D, d, L = max_batch, cfg.n_heads, self.D, cfg.d_model, cfg.n_layers
        self.B = B
        self.n_sites = 3 * L + 1
        off = 0
        self.flags_off = off
        off = _align(off + self.n_sites * MAX_CTAS * MAX_W * 4)
        self.q_off = off
        off = _align(off + B * H * D)
        self.ds_off = off
        off = _align(off + B * H * D // 32 * 8)
        self.parts_off = off
        off = _align(off + L * B * d * 4)
        self.cand_off = off
        off = _align(off + B * MAX_W * 8)
        # fused down-projection all-reduce: per-tile partial slots [src][tile][<=32 tokens] and flags
        self.ar_tiles = (d + 15) // 16
        self.arparts_off = off
        off = _align(off + MAX_W * self.ar_tiles * 4 * 128 * 4)
        self.arflags_off = off
        off = _align(off + self.ar_tiles * MAX_W * 4)
        self.nbytes = off
        self.buf = symm_mem.empty(self.nbytes, dtype=torch.uint8, device=device)
        self.buf.zero_()
        self.hdl = symm_mem.rendezvous(self.buf, group)
        self.peers = torch.tensor(list(self.hdl.buffer_ptrs), dtype=torch.int64)
        self.me = self.hdl.rank
        self.counters = torch.zeros(self.n_sites * MAX_CTAS, dtype=torch.int32, device=device)
        self.ar_epochs = torch.zeros(self.ar_tiles, dtype=torch.int32, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        torch.cuda.synchronize(device)
        dist.barrier(group=group)
        # views into the local symmetric buffer
        self.act_full = _ActView(self.buf[self.q_off:self.q_off + B * H * D].view(torch.int8).view(B, H * D),
                                 self.buf[self.ds_off:self.ds_off + B * H * D // 32 * 8].view(torch.float32)
                                 .view(B, H * D // 32, 2), H * D)
        from ..models.weights import head_assignment
        heads = head_assignment(cfg, self.rank, self.world)[0]
        if heads != list(range(heads[0], heads[0] + len(heads))):
            raise ValueError("P2P all-gather expects each rank's query heads to be contiguous")
        self.h0, self.nh = heads[0], len(heads)
        # attention writes this rank's heads at their global columns of the shared act buffer
        qflat = self.buf[self.q_off + self.h0 * D:self.q_off + B * H * D].view(torch.int8)
        dflat = self.buf[self.ds_off + self.h0 * D // 4:self.ds_off + B * H * D // 4].view(torch.float32)
        self.act_mine = _ActView(qflat, dflat, H * D)
        self.v_off = self.rank * self.Vl

    def check(self) -> int:
        """Device error word of the collective kernels (1 = a peer never arrived at a barrier)."""
        return int(self.err.item())

    # ---------------------------------------------------------------------------------
    def decode_attn_o(self, rn, i: int, B: int, bt, ctx, n_split: int) -> None:
        C, kv, D, H = ext(), rn.kv, self.D, self.cfg.n_heads
        K.decode_attention(rn.q[:B], kv.k[i], kv.v[i], bt, ctx, n_split, act=self.act_mine, workspace=rn.attn_ws,
                           tickets=rn.attn_tickets, ldo=H * D, window=self.cfg.layer_window(i),
                           **rn.cascade_args(B, self.cfg.layer_window(i)))
        # codes and (scale, sum) pairs of this rank's heads, pushed to every rank in one launch
        C.p2p_allgather_cols(self.peers, self.buf[self.q_off:], H * D, self.q_off, H * D, self.h0 * D, self.nh * D,
                             B, self.flags_off, 3 * i, self.me, self.counters, self.err, AG_CTAS,
                             self.buf[self.ds_off:], H * D // 4, self.ds_off, H * D // 4, self.h0 * D // 4,
                             self.nh * D // 4)
        K.count(1)
        K.gemv(rn.w.layers[i].o, self.act_full, B, rn.x[:B], None, K.EPI_ADD)

    def decode_down(self, rn, i: int, B: int) -> None:
        d = self.cfg.d_model
        w = rn.w.layers[i].down
        if w.tp is not None and B <= K.TGEMV_MAX_B:
            # one kernel: local K-split GEMV, per-tile push to every rank, rank-order sum, residual add
            K.gemv(w, rn.ffn_in, B, rn.x[:B], None, K.EPI_ADD,
                   ar=(self.peers, self.me, self.arparts_off, self.arflags_off, self.ar_epochs))
            return
        part_off = self.parts_off + i * self.B * d * 4
        part = self.buf[part_off:part_off + B * d * 4].view(torch.float32).view(B, d)
        K.gemv(rn.w.layers[i].down, rn.ffn_in, B, part, None, K.EPI_STORE)
        ext().p2p_allreduce_add(self.peers, part_off, rn.x[:B], B * d, self.flags_off, 3 * i + 2, self.me,
                                self.counters, self.err, AR_CTAS)
        K.count()

    def lm_head_greedy(self, rn, B: int) -> None:
        """Local vocab-shard logits, then the distributed first-index argmax into rn.next_ids."""
        K.gemv(rn.w.lm_head, rn.lm_in, B, self.logits_local[:B, :self.Vl_real], None, K.EPI_STORE)
        ext().p2p_argmax(self.peers, self.logits_local[:B], self.Vl_real, self.v_off, self.cand_off,
                         rn.next_ids[:B], B, self.flags_off, 3 * self.cfg.n_layers, self.me, self.counters, self.err)
        K.count()

    def reduce_partial(self, rn, i: int, B: int, fill) -> None:
        """x += sum over ranks of the partial fill() writes (MoE expert bands), via the P2P all-reduce."""
        d = self.cfg.d_model
        part_off = self.parts_off + i * self.B * d * 4
        part = self.buf[part_off:part_off + B * d * 4].view(torch.float32).view(B, d)
        fill(part)
        ext().p2p_allreduce_add(self.peers, part_off, rn.x[:B], B * d, self.flags_off, 3 * i + 2, self.me,
                                self.counters, self.err, AR_CTAS)
        K.count(2)
