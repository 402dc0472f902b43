"""Tensor-parallel decode with in-kernel peer-memory collectives (the fused path).

Every rank allocates one peer buffer (the same layout on every rank, each rank's buffer mapped into
every peer's address space over NVLink/NVSwitch: CUDA IPC handles by default, ``PeerBuffer``, with no
NVLink multicast object; ``FAK_P2P_MEM=symm`` uses torch symmetric memory instead) holding

* ``flags``   -- per-(site, CTA, source-rank) epoch flags of the cross-rank barriers;
* ``parts``   -- fp32 [B, d] partial-sum slots per (layer, projection) for the unfused fallback;
* ``cand``    -- argmax key lines (key and launch epoch in one 16-byte store) for greedy sampling
  over the vocab shards;
* ``arparts`` -- per-tile line slots of the all-reduce fused into the GEMV epilogue
  ([epoch parity][source rank][tile][<= 32 tokens]); each 16-byte line carries two values, each
  beside the launch epoch that marks it valid (no separate flags).

Both row-parallel projections of a decode layer -- the attention output projection (o_proj) and
the down projection -- all-reduce in their own GEMV epilogue: the warp that finishes a 16-row output
tile pushes the tile's partial to every rank, waits (bounded) for the other ranks' partials of that
tile and adds their rank-order sum to the replicated residual.  One kernel per projection, the
transfer of each tile overlapping the GEMV of the others, no separate collective launch and no
all-gather of the attention output (each rank streams only its slice of o_proj).  Batches above 32
tokens fall back to the GEMV + one-shot all-reduce kernel pair.  Greedy decoding ends with a
distributed argmax instead of gathering 152k logits.

Prefill can all-reduce both row-parallel projections (and the MoE expert sum) without NCCL
(``FAK_PREFILL_P2P=1``; NCCL's all-reduce is the default for prefill, measured faster): the tcgen05
GEMM's epilogue stores each 128 x 256 fp32 output tile into the owner rank's slot (owner = m-block
mod W, the reduce-scatter half; ``gemm_tc.cu`` ``G_RS``) and releases a tile flag, and the owner's
``k_p2p_rs_reduce`` adds the W partials to the residual and stores the rows into every rank's
residual (the all-gather half), which for that reason lives in the peer buffer (``prefill_x``).

Every wait is bounded (``spin_limit`` polls; 0 = the kernels' default of about a second) and writes
an error word the engine reads back with each step's tokens (``engine.Engine._collect``).
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from ..ops import kernels as K
from ..ops._ext import ext
from .tp import NcclTP

MAX_CTAS = 128
MAX_W = 8


def ar_slot_bytes(tiles: int) -> int:
    """Bytes of the fused all-reduce's line slots for ``tiles`` 16-row output tiles: two epoch
    parities x MAX_W source ranks x 4 token tiles x 32 lanes x two 16-byte lines."""
    return 2 * MAX_W * tiles * 4 * 32 * 32
AR_CTAS = 16
AG_CTAS = 16
RS_CTAS = 128


def _align(n: int, a: int = 256) -> int:
    return (n + a - 1) // a * a


class PeerBuffer:
    """A zeroed device buffer on every rank, each mapped into every other rank through a CUDA IPC
    handle (plain peer mappings, no multicast object).  ``buf``: this rank's buffer as a uint8 tensor;
    ``ptrs``: every rank's buffer address in this process, in rank order."""

    def __init__(self, nbytes: int, group, device: torch.device):
        C = ext()
        self.dev = device.index if device.index is not None else torch.cuda.current_device()
        self.rank = dist.get_rank(group)
        self.group = group
        ptr, handle = C.ipc_alloc(nbytes, self.dev)
        handles: list = [None] * dist.get_world_size(group)
        dist.all_gather_object(handles, bytes(handle.numpy().tobytes()), group=group)
        self.ptrs = []
        for r, hb in enumerate(handles):
            self.ptrs.append(ptr if r == self.rank else
                             C.ipc_open(torch.frombuffer(bytearray(hb), dtype=torch.uint8), self.dev))
        self.own = ptr
        self.buf = C.ipc_view(ptr, nbytes, self.dev)
        self.closed = False

    def close(self) -> None:
        """Unmap the peers' buffers, then free this rank's (after every rank has unmapped it)."""
        if self.closed:
            return
        self.closed = True
        C = ext()
        torch.cuda.synchronize(self.dev)
        dist.barrier(group=self.group)
        for p in self.ptrs:
            if p != self.own:
                C.ipc_close(p)
        dist.barrier(group=self.group)
        self.buf = None
        C.ipc_free(self.own)


class P2PTP(NcclTP):
    def __init__(self, group, weights, max_batch: int, device, spin_limit: int = 0, max_prefill_tokens: int = 0):
        super().__init__(group, weights, max_batch, device)
        cfg = self.cfg
        if self.world > MAX_W:
            raise ValueError(f"P2P collectives support up to {MAX_W} ranks")
        B, d, L = max_batch, cfg.d_model, cfg.n_layers
        self.B = B
        self.spin_limit = int(spin_limit)
        self.n_sites = 3 * L + 3   # per layer 3, the two LM-head sites, the prefill all-reduce's end barrier
        off = 0
        self.flags_off = off
        off = _align(off + self.n_sites * MAX_CTAS * MAX_W * 4)
        self.parts_off = off
        off = _align(off + 2 * L * B * d * 4)
        # greedy argmax: per-row key lines [2 parities][MAX_CTAS rows][MAX_W sources] x 16 B
        self.cand_off = off
        off = _align(off + 2 * MAX_CTAS * MAX_W * 16)
        # fused all-reduce: per-tile line slots [parity][src][tile][<= 4 n8 tiles][32 lanes] x 2 x 16 B,
        # each 16-byte line two (value, epoch) pairs
        self.ar_tiles = (d + 15) // 16
        self.arparts_off = off
        off = _align(off + ar_slot_bytes(self.ar_tiles))
        # sampled steps: full-vocabulary logit rows [B, W * Vl], rank r's shard at columns [r Vl, (r+1) Vl)
        self.lg_ok = self.Vl % 4 == 0
        self.lg_off = off
        off = _align(off + (B * self.world * self.Vl * 4 if self.lg_ok else 0))
        # MoE combine fused with the expert-parallel all-reduce: [2 layer parities][W][B * d] partials
        self.moe_off = off
        off = _align(off + (2 * self.world * B * d * 4 if cfg.is_moe else 0))
        # prefill all-reduce: the residual [T, d], partial slots [W][MR][d] (MR rows of owned
        # 128-row m-blocks per source rank) and tile flags [m-block][256-column block][MAX_W]
        Tp = max(0, int(max_prefill_tokens))
        # the fused prefill all-reduce is opt-in: at TP=2 on Qwen2.5-7B it measured TTFT p50 30.5-30.9 ms
        # against 28.6 ms with NCCL's all-reduce for the same turns
        self.pf_fused = Tp > 0 and d % 4 == 0 and os.environ.get("FAK_PREFILL_P2P", "0") == "1"
        Tp = Tp if self.pf_fused else 0
        n_m, n_n = -(-Tp // 128), -(-d // 256)
        self.pf_T, self.pf_MR = Tp, -(-n_m // self.world) * 128
        self.pf_x_off = off
        off = _align(off + Tp * d * 4)
        self.pf_parts_off = off
        off = _align(off + (self.world * self.pf_MR * d * 4 if Tp else 0))
        self.pf_flags_off = off
        off = _align(off + n_m * n_n * MAX_W * 4)
        self.pf_epoch = 0
        # sequence-parallel prefill: this rank's normalised rows [MR, d] bf16 (read by every rank's
        # column-parallel GEMM) and the per-m-block release flags the owners push to every rank
        self.sp = self.pf_fused and not cfg.is_moe and cfg.d_model % 128 == 0 and \
            os.environ.get("FAK_PREFILL_SP", "0") == "1"
        self.sp_shard_off = off
        off = _align(off + (self.pf_MR * d * 2 if self.sp else 0))
        self.sp_flags_off = off
        off = _align(off + (n_m * 4 if self.sp else 0))
        self.sp_epoch = 0
        self._sp_x = None
        self.nbytes = off
        self.mem = None
        if os.environ.get("FAK_P2P_MEM", "ipc") == "symm":
            import torch.distributed._symmetric_memory as symm_mem
            self.buf = symm_mem.empty(self.nbytes, dtype=torch.uint8, device=device)
            self.buf.zero_()
            hdl = symm_mem.rendezvous(self.buf, group)
            self.peers = torch.tensor(list(hdl.buffer_ptrs), dtype=torch.int64)
            self.me = hdl.rank
        else:
            self.mem = PeerBuffer(self.nbytes, group, torch.device(device))
            self.buf = self.mem.buf
            self.peers = torch.tensor(self.mem.ptrs, dtype=torch.int64)
            self.me = self.rank
        self.counters = torch.zeros(self.n_sites * MAX_CTAS, dtype=torch.int32, device=device)
        self.ar_epochs = torch.zeros(self.ar_tiles, dtype=torch.int32, device=device)
        self.argmax_epochs = torch.zeros(MAX_CTAS, dtype=torch.int32, device=device)
        self.argmax_ws = K.argmax_workspace(device, MAX_CTAS)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)   # replaced by the runner's status word
        if self.lg_ok:
            self._rows().fill_(float("-inf"))     # shard tails past the real vocabulary stay -inf
        torch.cuda.synchronize(device)
        dist.barrier(group=group)
        self.v_off = self.rank * self.Vl

    def close(self) -> None:
        """Release the peer buffers (every rank, after its last step)."""
        if self.mem is not None:
            self.mem.close()

    def check(self) -> int:
        """Device error word of the collective kernels (1 = a peer never arrived at a barrier)."""
        return int(self.err.item())

    def _ar(self) -> tuple:
        return (self.peers, self.me, self.arparts_off, self.ar_epochs, self.spin_limit)

    def _part(self, i: int, which: int, B: int) -> tuple[int, torch.Tensor]:
        d = self.cfg.d_model
        off = self.parts_off + (2 * i + which) * self.B * d * 4
        return off, self.buf[off:off + B * d * 4].view(torch.float32).view(B, d)

    def _row_parallel(self, rn, w, act, B: int, i: int, which: int) -> None:
        """x += sum over ranks of W_local . act (a row-parallel projection), fused when it can be."""
        if w.tp is not None and B <= K.TGEMV_MAX_B:
            # one kernel: local K-split GEMV, per-tile push to every rank, rank-order sum, residual add
            K.gemv(w, act, B, rn.x[:B], None, K.EPI_ADD, ar=self._ar())
            return
        off, part = self._part(i, which, B)
        K.gemv(w, act, B, part, None, K.EPI_STORE)
        ext().p2p_allreduce_add(self.peers, off, rn.x[:B], B * self.cfg.d_model, self.flags_off, 3 * i + 1 + which,
                                self.me, self.counters, self.err, AR_CTAS, self.spin_limit)
        K.count()

    # ---------------------------------------------------------------------------------
    def decode_attn_o(self, rn, i: int, B: int, bt, ctx, n_split: int) -> None:
        self.attention(rn, i, B, bt, ctx, n_split)
        self._row_parallel(rn, rn.w.layers[i].o, rn.act_attn, B, i, 0)

    def decode_down(self, rn, i: int, B: int) -> None:
        self._row_parallel(rn, rn.w.layers[i].down, rn.ffn_in, B, i, 1)

    def _rows(self) -> torch.Tensor:
        n = self.B * self.world * self.Vl
        return self.buf[self.lg_off:self.lg_off + 4 * n].view(torch.float32).view(self.B, self.world * self.Vl)

    def lm_head_rows(self, rn, B: int) -> tuple[torch.Tensor, int]:
        """Full logit rows for the device sampler: this rank's vocab shard written into its columns of
        the gathered rows, then pushed to every rank by the in-kernel all-gather (no NCCL); every rank
        then samples the same rows and draws the same tokens."""
        if not self.lg_ok:
            self.lm_head(rn, B)
            return rn.logits[:B], self.cfg.vocab_size
        rows = self._rows()
        c0 = self.rank * self.Vl
        K.gemv(rn.w.lm_head, rn.lm_in, B, rows[:B, c0:c0 + self.Vl_real], None, K.EPI_STORE)
        ld = self.world * self.Vl * 4
        ext().p2p_allgather_cols(self.peers, self.buf[self.lg_off:], ld, self.lg_off, ld, c0 * 4, self.Vl * 4, B,
                                 self.flags_off, 3 * self.cfg.n_layers + 1, self.me, self.counters, self.err, AG_CTAS,
                                 spin_limit=self.spin_limit)
        K.count()
        return rows[:B], self.world * self.Vl

    def lm_head_greedy(self, rn, B: int) -> None:
        """Local vocab-shard logits, then the distributed first-index argmax into rn.next_ids."""
        K.gemv(rn.w.lm_head, rn.lm_in, B, self.logits_local[:B, :self.Vl_real], None, K.EPI_STORE)
        ext().p2p_argmax(self.peers, self.logits_local[:B], self.Vl_real, self.v_off, self.cand_off,
                         rn.next_ids[:B], B, self.argmax_ws[0], self.argmax_ws[1], self.argmax_epochs, self.me,
                         self.err, self.spin_limit)
        K.count()

    def moe_combine(self, rn, i: int, B: int, st) -> None:
        """x += sum over ranks of this rank's router-weighted expert outputs: one kernel (combine,
        push to every rank, bounded barrier, rank-order sum)."""
        ext().p2p_moe_combine_ar(self.peers, st.out, st.ids[:B], st.wts[:B], st.k, st.e0, st.E_local, rn.x[:B], B,
                                 self.moe_off, i & 1, self.flags_off, 3 * i + 2, self.me, self.counters, self.err,
                                 AR_CTAS * 2, self.spin_limit)
        K.count()

    # ---- prefill ----------------------------------------------------------------------
    def prefill_x(self, T: int) -> torch.Tensor | None:
        """The prefill residual [T, d] fp32 inside this rank's peer buffer (the fused all-reduce
        stores reduced rows into every rank's copy), or None when the fused prefill path is off."""
        if not self.pf_fused or T > self.pf_T:
            return None
        d = self.cfg.d_model
        return self.buf[self.pf_x_off:self.pf_x_off + T * d * 4].view(torch.float32).view(T, d)

    def _pf_ok(self, x: torch.Tensor) -> bool:
        return (self.pf_fused and x.shape[0] <= self.pf_T and
                x.data_ptr() == self.buf.data_ptr() + self.pf_x_off and x.is_contiguous())

    def _pf_reduce(self, T: int) -> None:
        ext().p2p_rs_reduce(self.peers, self.pf_parts_off, self.pf_flags_off, self.pf_x_off, T, self.cfg.d_model,
                            self.pf_MR, self.me, self.pf_epoch, self.flags_off, self.n_sites - 1, self.counters,
                            self.err, RS_CTAS, self.spin_limit)

    def _pf_gemm_ar(self, a: torch.Tensor, w: torch.Tensor, x: torch.Tensor) -> None:
        """x += all-reduce(a . w^T): the GEMM pushes its tiles to their owners, the owners reduce
        and broadcast."""
        if a.shape[0] != x.shape[0] or w.shape[0] != self.cfg.d_model:
            raise ValueError("prefill all-reduce: the slots hold [tokens, d_model] partials")
        self.pf_epoch += 1
        ext().gemm_bf16_rs(a, w, self.peers, self.me, self.pf_parts_off, self.pf_flags_off, self.pf_MR,
                           self.pf_epoch, self.err)
        self._pf_reduce(x.shape[0])
        K.count(2)

    def prefill_attn_o(self, rn, i: int, ab: torch.Tensor, x: torch.Tensor) -> None:
        if not self._pf_ok(x):
            return super().prefill_attn_o(rn, i, ab, x)
        self._pf_gemm_ar(ab, self.o_dense_local(rn, i), x)

    def prefill_down(self, rn, i: int, hb2: torch.Tensor, x: torch.Tensor) -> None:
        if not self._pf_ok(x):
            return super().prefill_down(rn, i, hb2, x)
        self._pf_gemm_ar(hb2, rn.w.layers[i].down.dense(), x)

    def prefill_reduce(self, part: torch.Tensor, x: torch.Tensor) -> None:
        if not self._pf_ok(x):
            return super().prefill_reduce(part, x)
        if part.shape != x.shape:
            raise ValueError("prefill all-reduce: partial and residual shapes differ")
        self.pf_epoch += 1
        ext().p2p_rs_push(self.peers, part.contiguous(), self.pf_MR, self.pf_parts_off, self.pf_flags_off, self.me,
                          self.pf_epoch)
        self._pf_reduce(x.shape[0])
        K.count(2)

    # ---- sequence-parallel prefill ----------------------------------------------------
    def sp_ok(self, T: int) -> bool:
        return self.sp and 0 < T <= self.pf_T

    def sp_begin(self, T: int) -> tuple[torch.Tensor, torch.Tensor, int]:
        """(the owned-rows residual [MR, d] fp32, the global row of each of its rows (-1: padding),
        how many of its rows are real).  Rank me owns 128-row blocks me, me + W, ..."""
        d, W, MR = self.cfg.d_model, self.world, self.pf_MR
        if self._sp_x is None:
            self._sp_x = torch.zeros(MR, d, dtype=torch.float32, device=self.buf.device)
        n_m = -(-T // 128)
        rows = torch.full((MR,), -1, dtype=torch.int64)
        valid = 0
        for k, mb in enumerate(range(self.me, n_m, W)):
            n = min(128, T - mb * 128)
            rows[k * 128:k * 128 + n] = torch.arange(mb * 128, mb * 128 + n)
            valid = k * 128 + n
        return self._sp_x, rows.to(self.buf.device, non_blocking=True), valid

    def sp_norm(self, x: torch.Tensor, gamma: torch.Tensor, eps: float, valid: int) -> None:
        """RMSNorm of the owned rows into this rank's bf16 shard; each block's flag goes to every rank."""
        self.sp_epoch += 1
        ext().sp_rmsnorm_shard(self.peers, x, gamma, eps, valid, self.sp_shard_off, self.sp_flags_off, self.me,
                               self.sp_epoch)
        K.count()

    def sp_gemm(self, T: int, w: torch.Tensor, out: torch.Tensor, epi: int, bias) -> None:
        """out (op)= gathered-normalised-rows . w^T: each m-block of A read from its owner's shard."""
        ext().gemm_bf16_ag(T, w, out, self.peers, self.me, self.sp_shard_off, self.pf_MR, self.sp_flags_off,
                           self.sp_epoch, self.spin_limit, bias, epi, self.err)
        K.count()

    def sp_rs(self, a: torch.Tensor, w: torch.Tensor, x: torch.Tensor) -> None:
        """Owned rows += their slice of sum over ranks of a . w^T (reduce-scatter in the GEMM epilogue,
        the owner's sum into its compacted rows, no broadcast)."""
        if w.shape[0] != self.cfg.d_model:
            raise ValueError("sequence-parallel reduce: the slots hold [tokens, d_model] partials")
        T = a.shape[0]
        self.pf_epoch += 1
        ext().gemm_bf16_rs(a, w, self.peers, self.me, self.pf_parts_off, self.pf_flags_off, self.pf_MR,
                           self.pf_epoch, self.err)
        ext().p2p_rs_reduce(self.peers, self.pf_parts_off, self.pf_flags_off, self.pf_x_off, T, self.cfg.d_model,
                            self.pf_MR, self.me, self.pf_epoch, self.flags_off, self.n_sites - 1, self.counters,
                            self.err, RS_CTAS, self.spin_limit, x)
        K.count(2)

    def sp_rows(self, x: torch.Tensor, own_rows: torch.Tensor, last_idx: torch.Tensor) -> torch.Tensor:
        """[S, d]: the residual rows last_idx (global rows) gathered from their owners, through the
        in-kernel all-reduce (each rank contributes the rows it owns, zeros elsewhere)."""
        S, d = last_idx.numel(), self.cfg.d_model
        if S > self.B:
            raise ValueError(f"sequence-parallel prefill: {S} sequences in a chunk (at most {self.B})")
        loc = torch.full((self.pf_T + 128,), -1, dtype=torch.int64, device=x.device)
        real = own_rows >= 0
        loc[own_rows[real]] = torch.nonzero(real).flatten()
        li = loc[last_idx.long()]
        off, part = self._part(0, 0, S)
        part.copy_(torch.where((li >= 0)[:, None], x[li.clamp(min=0)], torch.zeros((), device=x.device)))
        out = torch.zeros(S, d, dtype=torch.float32, device=x.device)
        ext().p2p_allreduce_add(self.peers, off, out, S * d, self.flags_off, self.n_sites - 1, self.me, self.counters,
                                self.err, AR_CTAS, self.spin_limit)
        K.count(4)
        return out

    def reduce_partial(self, rn, i: int, B: int, fill) -> None:
        """x += sum over ranks of the partial fill() writes (MoE expert bands), via the P2P all-reduce."""
        off, part = self._part(i, 1, B)
        fill(part)
        ext().p2p_allreduce_add(self.peers, off, rn.x[:B], B * self.cfg.d_model, self.flags_off, 3 * i + 2, self.me,
                                self.counters, self.err, AR_CTAS, self.spin_limit)
        K.count(2)
