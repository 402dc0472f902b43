"""Forward passes of the dense Llama/Qwen2/Qwen3 and Qwen3-MoE decoders on the GPU.

Two entry points, both over the paged KV cache:

``decode``   B sequences advance one token.  Per layer: RMSNorm+int8 activation quant,
             q/k/v GEMV (+bias), RoPE (+q/k norm) with the K/V append into the pages,
             split-KV paged attention whose merge writes the o_proj input already
             quantized, o_proj GEMV accumulating into the fp32 residual, RMSNorm+quant,
             gate/up GEMV with a SwiGLU epilogue, quant, down GEMV accumulating into the
             residual.  The whole step is captured as one CUDA graph per batch bucket.
``prefill``  a packed chunk of new tokens from several sequences (ragged), each attending
             to its cached prefix + itself; bf16 activations through tensor-core GEMMs.

The reference runs the same per-token sequence of ops one kernel per op on one stream
(internal/model/hal.go:269-439, tokenHALOutput) and prefills with a per-token loop
(hal.go:522-534); batched decode shares one weight stream across lanes
(internal/model/batch_step.go:7).  With tensor parallelism the ``collectives`` object
supplies the gathers/reductions between the GEMVs (parallel/tp.py).
"""
from __future__ import annotations

import dataclasses
import math
import os

import torch

from ..config import ModelConfig
from ..ops import kernels as K
from .weights import ModelWeights


def rope_tables(max_pos: int, head_dim: int, theta: float, device, scaling=None, trained_context: int | None = None
                ) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin [max_pos, head_dim/2] (fp32, float64 angles; scaled RoPE resolved for the trained context)."""
    from .rope import cos_sin
    c, s = cos_sin(torch.arange(max_pos), head_dim, theta, scaling, trained_context)
    return c.to(device).contiguous(), s.to(device).contiguous()


@dataclasses.dataclass
class KVCache:
    k: torch.Tensor  # [L, P, Hkv_local, 16, D] bf16
    v: torch.Tensor

    @classmethod
    def allocate(cls, n_layers: int, n_pages: int, n_kv: int, head_dim: int, device, page_size: int = 16
                 ) -> "KVCache":
        shape = (n_layers, n_pages, n_kv, page_size, head_dim)
        return cls(torch.zeros(shape, dtype=torch.bfloat16, device=device),
                   torch.zeros(shape, dtype=torch.bfloat16, device=device))

    @property
    def n_pages(self) -> int:
        return self.k.shape[1]

    @staticmethod
    def bytes_per_page(n_layers: int, n_kv: int, head_dim: int, page_size: int = 16) -> int:
        return 2 * n_layers * n_kv * page_size * head_dim * 2


@dataclasses.dataclass
class PrefillMeta:
    """Packed ragged chunk description (all int32 device tensors): 64-query tiles for the mma.sync
    kernel and 128-query tiles (``tile128_*``) for the tcgen05 kernel."""
    tile_seq: torch.Tensor
    tile_q0: torch.Tensor
    seq_qoff: torch.Tensor
    seq_qlen: torch.Tensor
    seq_pos0: torch.Tensor
    n_tiles: int
    tile128_seq: torch.Tensor | None = None
    tile128_q0: torch.Tensor | None = None
    n_tiles128: int = 0

    @classmethod
    def build(cls, qlens: list[int], pos0s: list[int], device) -> "PrefillMeta":
        tile_seq, tile_q0, off, offs = [], [], 0, []
        t128_seq, t128_q0 = [], []
        for s, ql in enumerate(qlens):
            offs.append(off)
            for q0 in range(0, ql, 64):
                tile_seq.append(s)
                tile_q0.append(q0)
            for q0 in range(0, ql, 128):
                t128_seq.append(s)
                t128_q0.append(q0)
            off += ql
        mk = lambda a: torch.tensor(a, dtype=torch.int32).to(device, non_blocking=True)
        return cls(mk(tile_seq), mk(tile_q0), mk(offs), mk(qlens), mk(pos0s), len(tile_seq),
                   mk(t128_seq), mk(t128_q0), len(t128_seq))


class ModelRunner:
    def __init__(self, weights: ModelWeights, kv: KVCache, max_batch: int = 64, max_prefill_tokens: int = 4096,
                 max_context: int | None = None, collectives=None, fused_activations: bool = False,
                 attention_merge: bool = False, l2_prefetch: bool = False, cascade_attention: bool = True,
                 expert_offload=None):
        self.w = weights
        # models.moe_offload.ExpertOffload when the MoE experts live in host memory (their FFNs on the CPU)
        self.expert_offload = expert_offload
        self.cfg: ModelConfig = weights.cfg
        self.kv = kv
        self.coll = collectives
        cfg = self.cfg
        dev = kv.k.device
        self.device = dev
        self.max_batch = max_batch
        self.max_prefill = max_prefill_tokens
        self.max_context = max_context or cfg.max_context
        self.Hq = weights.n_q_local
        self.Hkv = weights.n_kv_local
        self.D = cfg.head_dim
        self.qkv_dim = (self.Hq + 2 * self.Hkv) * self.D
        f0, f1 = weights.ffn_slice
        self.ffn_local = (f1 - f0) if not cfg.is_moe else cfg.expert_ffn_dim
        self.cos, self.sin = rope_tables(self.max_context, self.D, cfg.rope_theta, dev, cfg.rope_scaling,
                                         cfg.max_context)
        B, d = max_batch, cfg.d_model
        # decode buffers (static: CUDA graphs capture their addresses)
        self.x = torch.zeros(B, d, dtype=torch.float32, device=dev)
        self.qkv = torch.zeros(B, self.qkv_dim, dtype=torch.float32, device=dev)
        self.q = torch.zeros(B, self.Hq, self.D, dtype=torch.float32, device=dev)
        self.h = torch.zeros(B, max(self.ffn_local, 32), dtype=torch.float32, device=dev)
        self.tmp = torch.zeros(B, d, dtype=torch.float32, device=dev)   # sandwich norms: projection outputs
        # gated FFN epilogue of the gate/up GEMV and GEMM: SwiGLU or GEGLU (GELU-tanh)
        self.gated_epi = K.EPI_GEGLU if cfg.act == "gelu_tanh" else K.EPI_SWIGLU
        if cfg.sandwich_norms and collectives is not None:
            raise NotImplementedError("sandwich-norm models (Gemma-2) run on one GPU per replica")
        gap = cfg.device_gap()
        if gap:
            raise NotImplementedError(f"{gap}; run it on the fp32 reference model (models.reference.ReferenceModel)")
        # activations quantized by quant_act feed the GEMVs with one scale per 256 columns when every
        # matrix that reads them is Q4_K / Q6_K (their integer-accumulating path); other formats gain
        # nothing from the coarser scale and keep one per 32 (so does FAK_UNIT_SCALE=0)
        unit_ok = os.environ.get("FAK_UNIT_SCALE", "1") != "0"

        def unit_for(mats) -> bool:
            return unit_ok and all(m is not None and m.qtype in (12, 14) for m in mats)   # Q4_K, Q6_K
        dense_layers = [L for L in weights.layers if getattr(L, "gate_up", None) is not None]
        unit_d = unit_for([sg for L in weights.layers for sg, _ in L.qkv] + [L.gate_up for L in dense_layers]) \
            and not cfg.is_moe
        unit_f = unit_for([L.down for L in dense_layers]) and bool(dense_layers)
        self.act_d = K.ActQ(B, d, dev, unit=unit_d)
        # o_proj input: this rank's slice [a0, a1) of the attention output columns (all of them on one
        # GPU); under TP the columns of other ranks' heads inside the slice stay zero
        a0, a1, _, _ = weights.o_cols if weights.o_cols[1] else (0, cfg.n_heads * self.D, 0, 0)
        self.act_attn = K.ActQ(B, a1 - a0, dev)
        self.act_ffn = K.ActQ(B, max(self.ffn_local, 32), dev, unit=unit_f)
        # decode GEMV inputs: activations quantized by a separate kernel (default), or fp32 sources
        # the GEMV normalises and quantizes itself (fused_activations: fewer launches, but every CTA
        # repeats the row's quantization; measured 0.14 ms/step slower on Qwen2.5-7B B=5).
        # attention_merge merges the attention splits in the last split's CTA instead of a combine
        # kernel (one CTA then reads all the partials of its heads: a long tail, 0.7 ms/step slower).
        self.fused_act = fused_activations
        # q|k and v in different block formats: one pair launch of the GEMV instead of two
        self.qkv_pair = os.environ.get("FAK_QKV_PAIR", "1") != "0"
        self.attn_merge = attention_merge
        self.l2_prefetch = l2_prefetch
        self.ffn_in = K.FAct(self.h) if self.fused_act else self.act_ffn   # SwiGLU output -> down projection
        self.lm_in = K.FAct(self.x) if self.fused_act else self.act_d      # final norm -> LM head
        self.logits = torch.zeros(B, cfg.vocab_size, dtype=torch.float32, device=dev)
        # step status, read back by the host in one copy: the sampled ids of every lane, the kernels'
        # error word (bounded waits that expired, out-of-range ids) and the collectives' error word
        self.status = torch.zeros(B + 2, dtype=torch.int32, device=dev)
        self.next_ids = self.status[:B]
        self.err = self.status[B:B + 1]
        if collectives is not None and hasattr(collectives, "err"):
            collectives.err = self.status[B + 1:B + 2]
        K.register_error_word(dev, self.err)
        # device sampler (sampled decode steps): per-lane parameter rows, the batch's logit-bias lists
        # and each lane's generated-token counts (frequency / presence penalties)
        from ..engine.sampling import MAX_BIAS
        self.samp_params = torch.zeros(B, 10, dtype=torch.int32, device=dev)
        self.bias_tok = torch.full((MAX_BIAS,), -1, dtype=torch.int32, device=dev)
        self.bias_val = torch.zeros(MAX_BIAS, dtype=torch.float32, device=dev)
        self.counts = torch.zeros(B, cfg.vocab_size, dtype=torch.int32, device=dev)
        # prefill attention on tcgen05 / TMEM (head dim 128, default scale, no soft-cap; windowed
        # layers and other shapes use the mma.sync kernel); FAK_PREFILL_ATTN=fa2 forces the latter
        self.tc_prefill_attn = (self.D == 128 and cfg.attn_scale == 0 and cfg.attn_softcap == 0 and not cfg.attn_sinks
                                and os.environ.get("FAK_PREFILL_ATTN", "tc") != "fa2")
        if collectives is not None and (cfg.attn_out_bias or cfg.moe_bias):
            raise NotImplementedError("gpt-oss blocks run on one GPU per replica on the device path")
        n_sm = torch.cuda.get_device_properties(dev).multi_processor_count if dev.type == "cuda" else 148
        # decode attention: with dec_pps > 0 a split holds dec_pps pages (more for contexts past
        # dec_pps x 256 pages) and the grid has a split for every dec_pps pages of the longest
        # context; splits past a sequence's pages exit at once.  0: 16 splits spread over the pages.
        self.dec_pps = int(os.environ.get("FAK_DEC_PPS", "0"))
        max_pages = -(-self.max_context // 16)
        auto = min(256, -(-max_pages // self.dec_pps)) if self.dec_pps > 0 else 16
        self.n_split = int(os.environ.get("FAK_DEC_SPLITS", "0")) or auto
        self.max_split = max(64, self.n_split)
        if not 1 <= self.n_split <= 256:
            raise ValueError("decode attention splits must be in [1, 256]")
        # cascade attention: prefix splits of the shared pages (about 2.6 CTAs per SM at 4 KV heads)
        self.prefix_splits = max(16, min(128, (5 * n_sm) // (2 * max(1, self.Hkv))))
        b_casc = min(B, 64 // max(1, self.Hq // max(1, self.Hkv)))   # lanes a cascade step can hold
        slots = max(B * self.max_split, b_casc * (self.n_split + self.prefix_splits))
        self.attn_ws = torch.zeros(slots * self.Hq * (self.D + 2), dtype=torch.float32, device=dev)
        self.attn_tickets = torch.zeros(B * self.Hkv, dtype=torch.int32, device=dev)  # split-merge tickets
        # cascade attention: pages shared by every lane of the step (a radix-shared prefix) are
        # attended once for the whole batch; the count lives on the device so graphs stay valid
        self.cascade = cascade_attention
        self._casc_on = False          # the step being run / captured uses cascade attention
        self.min_shared_pages = 32     # below this many shared pages the plain path is faster
        self.shared_pages = torch.zeros(1, dtype=torch.int32, device=dev)

        # per-device kernel scratch, allocated here so no graph capture allocates it
        mats = [weights.lm_head] + [m for L in weights.layers
                                    for m in [s for s, _ in L.qkv] + [L.o, L.gate_up, L.down]]
        K.tgemv_workspace(dev, mats)
        K.argmax_workspace(dev, B)
        self._graphs: dict[int, tuple[torch.cuda.CUDAGraph, dict]] = {}
        self._graph_kernels: dict[int, int] = {}
        # static decode inputs shared by every graph bucket (graphs capture their addresses): rows
        # ids / pos / slot / ctx of ``vec`` and the block table, one row per lane.  Between steps of
        # the device-resident decode loop they hold the lanes' state (Engine._run_decode_async)
        self._vec: torch.Tensor | None = None
        self._bt: torch.Tensor | None = None

    # ------------------------------------------------------------------------------------
    def n_split_for(self, B: int) -> int:
        """Context splits of the decode attention.  Independent of B on purpose: a sequence's
        attention then reduces in the same order whatever batch it runs in, so batched decode
        is bit-identical to serial decode.  The kernel spreads the live pages evenly over the
        splits, so short contexts just leave some splits empty.  16 (``FAK_DEC_SPLITS`` overrides):
        with 3 resident CTAs per SM, 22 splits fill one wave at 5 lanes x 4 KV heads and measured
        faster on the attention alone (20.1 against 21.4 us at 5 x 9K tokens with an 8K shared
        prefix), but the whole decode step at 5 x 9K unshared tokens ran 2% slower with 22 on the
        same box (3.17 against 3.11 ms), so 16 stays."""
        return self.n_split

    def cascade_ok(self, B: int) -> bool:
        """Cascade attention can run for a B-lane step (its prefix kernel holds <= 64 query rows)."""
        return self.cascade and B >= 2 and B * (self.Hq // max(1, self.Hkv)) <= 64

    def cascade_args(self, B: int, window: int = 0) -> dict:
        """Arguments that turn on cascade attention in the step being run or captured (none when
        the step is a plain one or cascade cannot apply)."""
        if not self._casc_on or window > 0 or not self.cascade_ok(B):
            return {}
        return {"shared_pages": self.shared_pages, "prefix_splits": self.prefix_splits}

    def _pf(self, w):
        """Tile-packed weights of ``w`` to warm L2 with during the current kernel (or None)."""
        return w.tp if self.l2_prefetch and w is not None and w.tp is not None else None

    def _qkv_pair(self, L, xin, B: int) -> bool:
        """The two q|k|v segments of different block formats as one pair launch (False: not possible)."""
        (sa, oa), (sb, ob) = L.qkv
        bias = L.qkv_bias
        return K.gemv_pair(sa, sb, xin, B, self.qkv[:B, oa:oa + sa.rows], self.qkv[:B, ob:ob + sb.rows],
                           bias[oa:oa + sa.rows] if bias is not None else None,
                           bias[ob:ob + sb.rows] if bias is not None else None)

    def _layer_decode(self, i: int, B: int, pos, slot, bt, ctx, n_split: int) -> None:
        cfg, L, kv = self.cfg, self.w.layers[i], self.kv
        x = self.x[:B]
        nxt = self.w.layers[i + 1] if i + 1 < cfg.n_layers else None
        segs = L.qkv
        if self.fused_act:
            xin = K.FAct(x, L.attn_norm, cfg.rms_eps)  # RMSNorm + quantization inside the GEMV
        else:
            K.quant_act(x, self.act_d, L.attn_norm, cfg.rms_eps, prefetch=self._pf(segs[0][0]))
            xin = self.act_d
        if not (self.qkv_pair and len(segs) == 2 and self._qkv_pair(L, xin, B)):
            for j, (seg, off) in enumerate(segs):
                bias = L.qkv_bias[off:off + seg.rows] if L.qkv_bias is not None else None
                pf = segs[j + 1][0] if j + 1 < len(segs) else None
                K.gemv(seg, xin, B, self.qkv[:B, off:off + seg.rows], bias, K.EPI_STORE, prefetch=self._pf(pf))
        K.rope_kv(self.qkv[:B], pos, slot, self.cos, self.sin, self.Hq, self.Hkv, L.q_norm, L.k_norm, cfg.rms_eps,
                  self.q[:B], None, kv.k[i], kv.v[i])
        if self.coll is None:
            K.decode_attention(self.q[:B], kv.k[i], kv.v[i], bt, ctx, n_split, pages_per_split=max(1, self.dec_pps),
                               act=self.act_attn,
                               workspace=self.attn_ws, tickets=self.attn_tickets if self.attn_merge else None,
                               prefetch=self._pf(L.o), window=cfg.layer_window(i),
                               scale=cfg.attn_scale, softcap=cfg.attn_softcap, sinks=L.attn_sinks,
                               **self.cascade_args(B, cfg.layer_window(i)))
            if L.post_attn_norm is not None:   # sandwich norm: x += rmsnorm(o_proj(a))
                K.gemv(L.o, self.act_attn, B, self.tmp[:B], L.o_bias, K.EPI_STORE, prefetch=self._pf(L.gate_up))
                K.rmsnorm_add(self.tmp[:B], L.post_attn_norm, cfg.rms_eps, x)
            else:
                K.gemv(L.o, self.act_attn, B, x, L.o_bias, K.EPI_ADD, prefetch=self._pf(L.gate_up))
        else:
            self.coll.decode_attn_o(self, i, B, bt, ctx, n_split)
        if cfg.is_moe:
            K.quant_act(x, self.act_d, L.ffn_norm, cfg.rms_eps)
            from .moe import moe_decode
            moe_decode(self, i, B)
            return
        if self.fused_act:
            K.gemv(L.gate_up, K.FAct(x, L.ffn_norm, cfg.rms_eps), B, self.h[:B], None, self.gated_epi)
        else:
            K.quant_act(x, self.act_d, L.ffn_norm, cfg.rms_eps)
            K.gemv(L.gate_up, self.act_d, B, self.h[:B], None, self.gated_epi, prefetch=self._pf(L.down))
            K.quant_act(self.h[:B, :self.ffn_local], self.act_ffn)
        if self.coll is None:
            nxt_w = nxt.qkv[0][0] if nxt is not None else self.w.lm_head
            pf = self._pf(nxt_w) if nxt is not None else None
            if L.post_ffn_norm is not None:   # sandwich norm: x += rmsnorm(down(h))
                K.gemv(L.down, self.ffn_in, B, self.tmp[:B], None, K.EPI_STORE, prefetch=pf)
                K.rmsnorm_add(self.tmp[:B], L.post_ffn_norm, cfg.rms_eps, x)
            else:
                K.gemv(L.down, self.ffn_in, B, x, None, K.EPI_ADD, prefetch=pf)
        else:
            self.coll.decode_down(self, i, B)

    def decode_eager(self, ids, pos, slot, bt, ctx, B: int, greedy: bool = True, n_layers: int | None = None,
                     cascade: bool = False, sampled: bool = False) -> None:
        self._casc_on = cascade
        try:
            self._decode_eager(ids, pos, slot, bt, ctx, B, greedy, n_layers, sampled)
        finally:
            self._casc_on = False

    def _decode_eager(self, ids, pos, slot, bt, ctx, B: int, greedy: bool = True, n_layers: int | None = None,
                      sampled: bool = False) -> None:
        """One decode step for B lanes; results in self.logits[:B] / self.next_ids[:B].

        ``n_layers`` < cfg.n_layers runs only the first layers before the final norm and LM head:
        the early-exit draft model of self-speculative decoding (its KV pages are the target's).
        ``sampled``: every lane draws its token with the device sampler (``samp_params`` rows, greedy
        rows included), from the full logits (gathered across tensor-parallel ranks)."""
        cfg = self.cfg
        n_split = self.n_split_for(B)
        K.embed(self.w.embed, ids, self.x[:B], None, self.err, scale=cfg.embed_scale)
        for i in range(cfg.n_layers if n_layers is None else n_layers):
            self._layer_decode(i, B, pos, slot, bt, ctx, n_split)
        if self.fused_act:
            self.lm_in = K.FAct(self.x, self.w.final_norm, cfg.rms_eps)
        else:
            K.quant_act(self.x[:B], self.act_d, self.w.final_norm, cfg.rms_eps)
            self.lm_in = self.act_d
        if sampled:
            rows, V = self._lm_head_full(B)
            K.sample_rows(rows, V, self.samp_params[:B], self.bias_tok, self.bias_val, self.counts[:B],
                          self.next_ids[:B], B, cfg.final_softcap)
            return
        if greedy and self.coll is not None and hasattr(self.coll, "lm_head_greedy"):
            self.coll.lm_head_greedy(self, B)  # sharded logits -> distributed argmax, no logits gather
            return
        self._lm_head(B)
        if greedy:
            K.argmax(self.logits[:B], self.logits.shape[1], self.next_ids[:B])

    def _lm_head_full(self, B: int) -> tuple[torch.Tensor, int]:
        """Full-vocabulary logit rows [B, >=V] of the step and the column count to sample over."""
        if self.coll is not None and hasattr(self.coll, "lm_head_rows"):
            return self.coll.lm_head_rows(self, B)
        self._lm_head(B)
        return self.logits[:B], self.cfg.vocab_size

    def _lm_head(self, B: int) -> None:
        if self.coll is None:
            K.gemv(self.w.lm_head, self.lm_in, B, self.logits[:B], None, K.EPI_STORE)
        else:
            self.coll.lm_head(self, B)

    # ------------------------------------------------------------------------------------
    # CUDA graph per batch bucket
    # ------------------------------------------------------------------------------------
    def lane_state(self, bt_width: int) -> tuple[torch.Tensor, torch.Tensor]:
        """The shared static decode inputs: ``vec`` int32 [4, max_batch] (rows ids, pos, slot, ctx)
        and the block table int32 [max_batch, bt_width].  Idle lanes have slot -1 and ctx 1."""
        if self._vec is None:
            dev = self.device
            self._vec = torch.zeros(4, self.max_batch, dtype=torch.int32, device=dev)
            self._vec[2].fill_(-1)
            self._vec[3].fill_(1)
            self._bt = torch.zeros(self.max_batch, bt_width, dtype=torch.int32, device=dev)
        if self._bt.shape[1] != bt_width:
            raise ValueError(f"block-table width {bt_width} differs from the captured {self._bt.shape[1]}")
        return self._vec, self._bt

    def _static_inputs(self, B: int, bt_width: int) -> dict:
        vec, bt = self.lane_state(bt_width)
        return {"ids": vec[0, :B], "pos": vec[1, :B], "slot": vec[2, :B], "ctx": vec[3, :B], "bt": bt[:B]}

    def capture(self, B: int, bt_width: int, n_layers: int | None = None) -> None:
        """Capture the B-lane step: the plain variant, and (target model, cascade possible) the
        cascade variant replayed when the lanes share enough prefix pages."""
        st = self._static_inputs(B, bt_width)
        variants = [(False, False)]
        if n_layers is None:
            variants += [(True, False)] if self.cascade_ok(B) else []
            variants += [(False, True)]     # sampled lanes: the device sampler instead of the argmax
        for casc, samp in variants:
            # warm up (also triggers lazy cudaFuncSetAttribute) on a side stream, then capture
            s = torch.cuda.Stream(device=self.device)
            s.wait_stream(torch.cuda.current_stream(self.device))
            saved = self.samp_params[:B].clone()
            with torch.cuda.stream(s):
                self.decode_eager(st["ids"], st["pos"], st["slot"], st["bt"], st["ctx"], B, n_layers=n_layers,
                                  cascade=casc, sampled=samp)
            torch.cuda.current_stream(self.device).wait_stream(s)
            torch.cuda.synchronize(self.device)
            self.samp_params[:B].copy_(saved)      # the warm-up advanced the lanes' draw counters
            g = torch.cuda.CUDAGraph()
            before = K.launches()
            with torch.cuda.graph(g):
                self.decode_eager(st["ids"], st["pos"], st["slot"], st["bt"], st["ctx"], B, n_layers=n_layers,
                                  cascade=casc, sampled=samp)
                if n_layers is None:
                    # the step's tokens become the next step's inputs on the device (idle lanes stay idle)
                    K.decode_advance(self.next_ids, st["ids"], st["pos"], st["slot"], st["ctx"], st["bt"], B)
            key = (B, n_layers, casc, samp)
            self._graph_kernels[key] = K.launches() - before
            K._launches[0] = before
            self._graphs[key] = (g, st)

    def replay_resident(self, B: int, n_shared: int = 0, sampled: bool = False) -> None:
        """One decode step of the device-resident lanes [0, B) (their inputs already in the shared
        static buffers, lanes [B, bucket) idle); the graph ends by advancing the lanes' inputs.
        ``n_shared``: the lanes' common leading pages (``shared_pages`` already holds the count on
        the device); with at least ``min_shared_pages`` the cascade variant runs.  ``sampled``: the
        variant that draws every lane's token with the device sampler (``samp_params`` filled)."""
        casc = (not sampled and n_shared >= self.min_shared_pages
                and self.graph_bucket(B, None, True) is not None)
        bucket = self.graph_bucket(B, None, casc, sampled)
        if bucket is None:
            raise RuntimeError(f"no captured decode graph holds {B} lanes")
        g, _ = self._graphs[(bucket, None, casc, sampled)]
        g.replay()
        K.count(self._graph_kernels[(bucket, None, casc, sampled)])

    def graph_bucket(self, B: int, n_layers: int | None = None, cascade: bool = False,
                     sampled: bool = False) -> int | None:
        cands = [b for b, nl, c, sm in self._graphs if b >= B and nl == n_layers and c == cascade and sm == sampled]
        return min(cands) if cands else None

    def decode(self, ids, pos, slot, bt, ctx, B: int, use_graph: bool = True, n_layers: int | None = None,
               shared: torch.Tensor | None = None, n_shared: int = 0) -> torch.Tensor:
        """Decode one token for B lanes; returns next ids (device int32 [B]).  ``shared`` (int32 [1]
        on the device) / ``n_shared`` (the same count on the host): leading block-table pages that are
        the same physical pages in every lane and lie before every lane's current page; with at
        least ``min_shared_pages`` of them the step runs cascade attention."""
        casc = shared is not None and n_shared >= self.min_shared_pages and n_layers is None
        if casc:
            self.shared_pages.copy_(shared)
        bucket = None
        if use_graph:
            bucket = self.graph_bucket(B, n_layers, casc) if casc else None
            if bucket is None:
                casc, bucket = False, self.graph_bucket(B, n_layers, False)
        if bucket is None:
            self.decode_eager(ids, pos, slot, bt, ctx, B, n_layers=n_layers, cascade=casc and self.cascade_ok(B))
            return self.next_ids[:B]
        g, st = self._graphs[(bucket, n_layers, casc, False)]
        st["ids"][:B].copy_(ids)
        st["pos"][:B].copy_(pos)
        st["slot"][:B].copy_(slot)
        w = min(bt.shape[1], st["bt"].shape[1])
        st["bt"][:B, :w].copy_(bt[:, :w])
        st["ctx"][:B].copy_(ctx)
        if bucket > B:  # padding lanes: a 1-token context on page 0 of their own slot
            st["ctx"][B:].fill_(1)
            st["slot"][B:].fill_(-1)
        g.replay()
        K.count(self._graph_kernels[(bucket, n_layers, casc, False)])
        return self.next_ids[:B]

    # ------------------------------------------------------------------------------------
    # prefill
    # ------------------------------------------------------------------------------------
    def prefill(self, ids, pos, slot, bt, meta: PrefillMeta, last_idx: torch.Tensor) -> torch.Tensor:
        """Run a packed chunk; returns logits [S, V] for each sequence's last token (and next ids)."""
        cfg, dev = self.cfg, self.device
        T = ids.numel()
        d = cfg.d_model
        if self.coll is not None and getattr(self.coll, "sp_ok", lambda *_: False)(T):
            return self._prefill_sp(ids, pos, slot, bt, meta, last_idx)
        # under fused tensor parallelism the residual lives in the peer buffer (the prefill all-reduce
        # stores reduced rows into every rank's copy)
        x = self.coll.prefill_x(T) if self.coll is not None and hasattr(self.coll, "prefill_x") else None
        if x is None:
            x = torch.empty(T, d, dtype=torch.float32, device=dev)
        hb = torch.empty(T, d, dtype=torch.bfloat16, device=dev)
        qkv = torch.empty(T, self.qkv_dim, dtype=torch.float32, device=dev)
        qb = torch.empty(T, self.Hq, self.D, dtype=torch.bfloat16, device=dev)
        ab = torch.empty(T, self.Hq * self.D, dtype=torch.bfloat16, device=dev)
        K.embed(self.w.embed, ids, x, None, self.err, scale=cfg.embed_scale)
        tmp = torch.empty(T, d, dtype=torch.float32, device=dev) if cfg.sandwich_norms else None
        for i in range(cfg.n_layers):
            L = self.w.layers[i]
            K.rmsnorm_bf16(x, L.attn_norm, cfg.rms_eps, hb)
            for seg, off in L.qkv:
                bias = L.qkv_bias[off:off + seg.rows] if L.qkv_bias is not None else None
                K.gemm(hb, seg, qkv[:, off:off + seg.rows], K.EPI_STORE, bias)
            K.rope_kv(qkv, pos, slot, self.cos, self.sin, self.Hq, self.Hkv, L.q_norm, L.k_norm, cfg.rms_eps,
                      None, qb, self.kv.k[i], self.kv.v[i])
            if self.tc_prefill_attn and cfg.layer_window(i) <= 0:
                K.prefill_attention_tc(qb, self.kv.k, self.kv.v, i, bt, meta, ab, self.err)
            else:
                K.prefill_attention(qb, self.kv.k[i], self.kv.v[i], bt, meta, ab, cfg.layer_window(i),
                                    cfg.attn_scale, cfg.attn_softcap, L.attn_sinks)
            if self.coll is None and L.post_attn_norm is not None:
                K.gemm(ab, L.o, tmp, K.EPI_STORE, L.o_bias)
                K.rmsnorm_add(tmp, L.post_attn_norm, cfg.rms_eps, x)
            elif self.coll is None:
                K.gemm(ab, L.o, x, K.EPI_ADD, L.o_bias)
            else:
                self.coll.prefill_attn_o(self, i, ab, x)
            K.rmsnorm_bf16(x, L.ffn_norm, cfg.rms_eps, hb)
            if cfg.is_moe:
                from .moe import moe_prefill
                moe_prefill(self, i, hb, x)
                continue
            hb2 = torch.empty(T, self.ffn_local, dtype=torch.bfloat16, device=dev)   # the gated product, bf16
            K.gemm(hb, L.gate_up, hb2, self.gated_epi)
            if self.coll is None and L.post_ffn_norm is not None:
                K.gemm(hb2, L.down, tmp, K.EPI_STORE)
                K.rmsnorm_add(tmp, L.post_ffn_norm, cfg.rms_eps, x)
            elif self.coll is None:
                K.gemm(hb2, L.down, x, K.EPI_ADD)
            else:
                self.coll.prefill_down(self, i, hb2, x)
        return self._prefill_logits(x.index_select(0, last_idx.long()))

    def _prefill_logits(self, xl: torch.Tensor) -> torch.Tensor:
        """LM-head logits [S, V] of the chunk's last rows xl [S, d] (final norm inside the GEMV)."""
        cfg, dev = self.cfg, self.device
        S = xl.shape[0]
        logits = torch.empty(S, cfg.vocab_size, dtype=torch.float32, device=dev)
        for s0 in range(0, S, self.max_batch):
            s1 = min(S, s0 + self.max_batch)
            n = s1 - s0
            self.lm_in = K.FAct(xl[s0:s1], self.w.final_norm, cfg.rms_eps)
            if self.coll is None:
                K.gemv(self.w.lm_head, self.lm_in, n, logits[s0:s1], None, K.EPI_STORE)
            else:
                self.coll.lm_head_to(self, n, logits[s0:s1])
        return logits

    def _prefill_sp(self, ids, pos, slot, bt, meta: PrefillMeta, last_idx: torch.Tensor) -> torch.Tensor:
        """Sequence-parallel prefill under fused tensor parallelism (Megatron-SP).  The residual stays
        sharded by 128-row blocks (rank r owns blocks r, r + W, ...): each rank embeds and normalises
        only its rows, the column-parallel GEMMs (qkv, gate/up) gather their input blocks from the
        owners inside the GEMM, and the row-parallel ones (o_proj, down) reduce-scatter their output
        tiles to the owners, which add them to their rows -- no full-residual all-gather at all."""
        cfg, dev, coll = self.cfg, self.device, self.coll
        T = ids.numel()
        x, own_rows, valid = coll.sp_begin(T)
        K.embed(self.w.embed, ids.index_select(0, own_rows.clamp(min=0)), x, None, self.err, scale=cfg.embed_scale)
        qkv = torch.empty(T, self.qkv_dim, dtype=torch.float32, device=dev)
        qb = torch.empty(T, self.Hq, self.D, dtype=torch.bfloat16, device=dev)
        ab = torch.empty(T, self.Hq * self.D, dtype=torch.bfloat16, device=dev)
        for i in range(cfg.n_layers):
            L = self.w.layers[i]
            coll.sp_norm(x, L.attn_norm, cfg.rms_eps, valid)
            for seg, off in L.qkv:
                bias = L.qkv_bias[off:off + seg.rows] if L.qkv_bias is not None else None
                coll.sp_gemm(T, seg.dense(), qkv[:, off:off + seg.rows], K.EPI_STORE, bias)
            K.rope_kv(qkv, pos, slot, self.cos, self.sin, self.Hq, self.Hkv, L.q_norm, L.k_norm, cfg.rms_eps,
                      None, qb, self.kv.k[i], self.kv.v[i])
            if self.tc_prefill_attn and cfg.layer_window(i) <= 0:
                K.prefill_attention_tc(qb, self.kv.k, self.kv.v, i, bt, meta, ab, self.err)
            else:
                K.prefill_attention(qb, self.kv.k[i], self.kv.v[i], bt, meta, ab, cfg.layer_window(i),
                                    cfg.attn_scale, cfg.attn_softcap)
            coll.sp_rs(ab, coll.o_dense_local(self, i), x)
            coll.sp_norm(x, L.ffn_norm, cfg.rms_eps, valid)
            hb2 = torch.empty(T, self.ffn_local, dtype=torch.bfloat16, device=dev)
            coll.sp_gemm(T, L.gate_up.dense(), hb2, self.gated_epi, None)
            coll.sp_rs(hb2, L.down.dense(), x)
        return self._prefill_logits(coll.sp_rows(x, own_rows, last_idx))
