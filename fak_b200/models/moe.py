"""Mixture-of-experts FFN (Qwen3-MoE family) on the GPU, with expert parallelism.

Decode (graph-capturable, no host sync): router kernel (fused RMSNorm, fp32 logits, softmax,
top-k, renorm) -> deterministic grouping of (token, expert) pairs into <=8-pair chunks per local
expert -> grouped int8-MMA GEMV for gate/up with a SwiGLU epilogue -> activation quant -> grouped
GEMV for down -> weighted combine (fixed order).  Prefill gathers each local expert's tokens and
runs the tcgen05 bf16 GEMM on the expert's dequantized weights.

Expert parallelism: rank r of the tensor-parallel group holds a contiguous band of experts
(models.weights.expert_slice), computes the contributions of the pairs routed to its band and
the partial sums are all-reduced into the residual -- the reference's EP decode scheme
(replicated router, rank-local experts, dense partial all-reduce: internal/model/moe.go:523-553,
internal/model/expert_parallel.go:85-200).  Attention is head-parallel, so every rank holds every
token's activation and the "dispatch" is the local row gather in the grouped GEMV's staging; the
combine and the cross-rank reduction are one kernel on the fused path (``P2PTP.moe_combine``).
"""
from __future__ import annotations

import torch

from ..ops import kernels as K
from ..ops import quant as dq
from ..ops._ext import ext


class MoEState:
    def __init__(self, rn):
        cfg = rn.cfg
        L0 = rn.w.layers[0]
        self.k = cfg.n_experts_used
        self.E_local = len(L0.expert_ids)
        self.e0 = L0.expert_ids[0]
        dev = rn.device
        B = rn.max_batch
        P = B * self.k
        self.max_chunks = -(-P // 8) + self.E_local
        self.ids = torch.zeros(B, self.k, dtype=torch.int32, device=dev)
        self.wts = torch.zeros(B, self.k, dtype=torch.float32, device=dev)
        self.chunk_expert = torch.zeros(self.max_chunks, dtype=torch.int32, device=dev)
        self.chunk_pairs = torch.full((self.max_chunks * 8,), -1, dtype=torch.int32, device=dev)
        self.n_chunks = torch.zeros(1, dtype=torch.int32, device=dev)
        f, d = cfg.expert_ffn_dim, cfg.d_model
        self.h = torch.zeros(P, f, dtype=torch.float32, device=dev)
        self.act_h = K.ActQ(P, f, dev)
        self.out = torch.zeros(P, d, dtype=torch.float32, device=dev)
        self.partial = torch.zeros(B, d, dtype=torch.float32, device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)


def _state(rn) -> MoEState:
    st = getattr(rn, "_moe", None)
    if st is None:
        st = rn._moe = MoEState(rn)
    return st


def _gate_epi(cfg) -> int:
    """The gated epilogue of the experts: gpt-oss's clamped gate, else SwiGLU."""
    return K.EPI_OAI if cfg.swiglu_alpha else K.EPI_SWIGLU


def _route(rn, L, x: torch.Tensor, ids: torch.Tensor, wts: torch.Tensor) -> None:
    cfg = rn.cfg
    ext().moe_route(x, L.ffn_norm, cfg.rms_eps, L.router, cfg.n_experts_used, cfg.norm_topk_prob, ids, wts,
                    L.router_bias, 1 if cfg.router == "topk_softmax" else 0)


def _grouped_ffn(rn, L, st: MoEState, n_tok: int, act) -> None:
    C = ext()
    P = n_tok * st.k
    C.moe_group(st.ids[:n_tok], P, st.e0, st.E_local, st.max_chunks, st.chunk_expert, st.chunk_pairs, st.n_chunks)
    gu, dn = L.experts_gate_up, L.experts_down
    if gu.tp is not None and dn.tp is not None:
        # tile-packed experts: one CTA per chunk streams its expert's tiles through per-warp rings
        C.moe_tgemv(gu.tp, gu.qtype, gu.rows // st.E_local, gu.cols, act.q, act.ds, st.k, True,
                    st.chunk_expert, st.chunk_pairs, st.n_chunks, st.max_chunks, st.h, _gate_epi(rn.cfg), st.err,
                    L.experts_gate_up_bias)
        K.quant_act(st.h[:P], st.act_h)
        C.moe_tgemv(dn.tp, dn.qtype, dn.rows // st.E_local, dn.cols, st.act_h.q, st.act_h.ds, st.k, False,
                    st.chunk_expert, st.chunk_pairs, st.n_chunks, st.max_chunks, st.out, 0, st.err,
                    L.experts_down_bias)
    else:
        if L.experts_gate_up_bias is not None or rn.cfg.swiglu_alpha:
            raise NotImplementedError("biased / clamped-gate experts need tile-packed weights (widths % 256)")
        C.moe_qmmv(gu.buf, gu.qtype, gu.rows // st.E_local, gu.cols, gu.pitch, act.q, act.ds, st.k, True,
                   st.chunk_expert, st.chunk_pairs, st.n_chunks, st.max_chunks, st.h, 2, st.err)
        K.quant_act(st.h[:P], st.act_h)
        C.moe_qmmv(dn.buf, dn.qtype, dn.rows // st.E_local, dn.cols, dn.pitch, st.act_h.q, st.act_h.ds, st.k,
                   False, st.chunk_expert, st.chunk_pairs, st.n_chunks, st.max_chunks, st.out, 0, st.err)
    K.count(3)


def moe_decode(rn, i: int, B: int) -> None:
    if rn.expert_offload is not None:   # experts in host memory: their FFNs run on the CPU
        rn.expert_offload.decode(rn, i, B)
        return
    cfg, L, st = rn.cfg, rn.w.layers[i], _state(rn)
    C = ext()
    x = rn.x[:B]
    _route(rn, L, x, st.ids[:B], st.wts[:B])
    K.count()
    _grouped_ffn(rn, L, st, B, rn.act_d)
    if rn.coll is None:
        C.moe_combine(st.out, st.ids[:B], st.wts[:B], st.k, st.e0, st.E_local, x)
        K.count()
    elif hasattr(rn.coll, "moe_combine"):
        rn.coll.moe_combine(rn, i, B, st)      # combine fused with the all-reduce (one kernel)
    else:
        rn.coll.reduce_partial(rn, i, B, lambda part: (part.zero_(), C.moe_combine(
            st.out, st.ids[:B], st.wts[:B], st.k, st.e0, st.E_local, part)))


def moe_prefill(rn, i: int, hb: torch.Tensor, x: torch.Tensor) -> None:
    """Per-expert dense GEMMs over the gathered tokens of each local expert (host-side grouping)."""
    if rn.expert_offload is not None:
        rn.expert_offload.prefill(rn, i, x)
        return
    cfg, L = rn.cfg, rn.w.layers[i]
    C = ext()
    T = x.shape[0]
    k = cfg.n_experts_used
    ids = torch.empty(T, k, dtype=torch.int32, device=x.device)
    wts = torch.empty(T, k, dtype=torch.float32, device=x.device)
    _route(rn, L, x, ids, wts)
    e0, E_local = L.expert_ids[0], len(L.expert_ids)
    gu, dn = L.experts_gate_up, L.experts_down
    rows_gu, rows_dn = gu.rows // E_local, dn.rows // E_local
    f, d = cfg.expert_ffn_dim, cfg.d_model
    out = torch.zeros(T * k, d, dtype=torch.float32, device=x.device)
    flat = ids.view(-1).long()
    host_ids = flat.cpu()
    # bf16 copies of the local experts, made at the first prefill and kept (like the dense layers'
    # prefill copies): later prefills run the GEMMs without dequantizing
    dense = getattr(L, "_dense_experts", None)
    if dense is None:
        dense = L._dense_experts = [None] * E_local
    for el in range(E_local):
        pairs = (host_ids == e0 + el).nonzero().view(-1)
        if pairs.numel() == 0:
            continue
        pairs_d = pairs.to(x.device)
        a = hb.index_select(0, pairs_d // k).contiguous()
        if dense[el] is None:
            dense[el] = (dq.dequantize_rows(gu.buf[el * rows_gu * gu.pitch:], gu.qtype, rows_gu, gu.cols, gu.pitch,
                                            torch.bfloat16),
                         dq.dequantize_rows(dn.buf[el * rows_dn * dn.pitch:], dn.qtype, rows_dn, dn.cols, dn.pitch,
                                            torch.bfloat16))
        wg, wd = dense[el]
        bgu = L.experts_gate_up_bias[el * rows_gu:(el + 1) * rows_gu] if L.experts_gate_up_bias is not None else None
        bdn = L.experts_down_bias[el * d:(el + 1) * d] if L.experts_down_bias is not None else None
        h = torch.empty(a.shape[0], f, dtype=torch.bfloat16, device=x.device)   # the gated product, bf16
        K.gemm(a, wg, h, _gate_epi(cfg), bgu)
        o = torch.empty(a.shape[0], d, dtype=torch.float32, device=x.device)
        K.gemm(h, wd, o, K.EPI_STORE, bdn)
        out.index_copy_(0, pairs_d, o)
    if rn.coll is None:
        C.moe_combine(out, ids, wts, k, e0, E_local, x)
    else:
        part = torch.zeros_like(x)
        C.moe_combine(out, ids, wts, k, e0, E_local, part)
        rn.coll.prefill_reduce(part, x)
