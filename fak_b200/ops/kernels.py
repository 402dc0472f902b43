"""Thin typed wrappers over the sm_100a extension, plus the GEMM dispatch used by prefill."""
from __future__ import annotations

import torch

from ._ext import ext

EPI_STORE, EPI_ADD, EPI_SWIGLU, EPI_GEGLU = 0, 1, 2, 3
EPI_OAI = 4   # the gpt-oss clamped gate: (clamp(u, -7, 7) + 1) * min(g, 7) * sigmoid(1.702 min(g, 7))
GEMV_MAX_B = 8      # tokens per launch of the row-major kernels
TGEMV_MAX_B = 32    # tokens per launch of the tile-packed GEMV (4 MMA column tiles)

# kernel-launch accounting (the benchmark reports how many of this package's kernels ran)
_launches = [0]


def count(n: int = 1) -> None:
    _launches[0] += n


def launches() -> int:
    return _launches[0]


def reset_launches() -> None:
    _launches[0] = 0


# per-device error word the kernels report bounded-wait expiries into (ModelRunner registers its
# status word here, so the host reads it back with the step's tokens)
_err_word: dict = {}


def register_error_word(device, word: torch.Tensor | None) -> None:
    key = torch.device(device)
    if word is None:
        _err_word.pop(key, None)
    else:
        _err_word[key] = word


def error_word(device) -> torch.Tensor | None:
    return _err_word.get(torch.device(device))


def decode_advance(next_ids, ids, pos, slot, ctx, bt, B: int) -> None:
    """Next decode step's lane inputs from this step's tokens, on the device: ids <- next_ids,
    pos += 1, ctx = pos + 1, slot from the block table (lanes with slot < 0 stay idle)."""
    ext().decode_advance(next_ids, ids, pos, slot, ctx, bt, B)
    count()


def sample_rows(logits: torch.Tensor, V: int, params: torch.Tensor, bias_tok: torch.Tensor, bias_val: torch.Tensor,
                counts: torch.Tensor | None, out: torch.Tensor, B: int, softcap: float = 0.0) -> None:
    """One token per row of logits [B, >=V] (modified in place): soft-cap, penalties from ``counts``,
    clamped logit bias, temperature / top-k / top-p and a Philox draw keyed by each row's (seed, step);
    params int32 [B, 10] (engine.sampling.pack_params; the step word is advanced)."""
    ext().sample_rows(logits, V, params, bias_tok, bias_val, counts, out, B, softcap)
    count()


def scatter_i32(dst: torch.Tensor, idx_val: torch.Tensor, n: int) -> None:
    """dst.flatten()[idx_val[i, 0]] = idx_val[i, 1] for i < n (device tensors)."""
    ext().scatter_i32(dst, idx_val, n)
    count()


class ActQ:
    """int8-quantized activations: codes [B, K] and per-32 (scale, sum) [B, K/32, 2].

    ``unit``: the quantizer chooses one scale per 256 columns (stored in each of the unit's eight
    entries, the format unchanged), so Q4_K GEMVs take their integer-accumulating path; producers
    that fill the buffer some other way (the attention merge) leave it False."""

    def __init__(self, B: int, K: int, device, unit: bool = False):
        self.K = K
        self.unit = unit and K % 256 == 0
        self.q = torch.zeros(B, K, dtype=torch.int8, device=device)
        self.ds = torch.zeros(B, K // 32, 2, dtype=torch.float32, device=device)


class FAct:
    """fp32 activations [B, >=K] that the tile-packed GEMV normalises (RMSNorm with ``gamma``, when
    given) and quantizes itself while its weight copies are in flight -- no separate quantizer
    launch.  The matrix's column count is K."""

    def __init__(self, x: torch.Tensor, gamma: torch.Tensor | None = None, eps: float = 1e-6):
        self.x, self.gamma, self.eps = x, gamma, float(eps)


def quant_act(x: torch.Tensor, act: ActQ, gamma: torch.Tensor | None = None, eps: float = 1e-6,
              prefetch: torch.Tensor | None = None) -> None:
    """prefetch: a tensor (e.g. the next GEMV's tile-packed weights) to warm L2 with meanwhile."""
    ext().quant_act_wide(x, gamma, eps, act.q, act.ds, prefetch, getattr(act, "unit", False))
    count()


# below this many tokens the CUDA-core dp4a GEMV is cheaper than the int8 MMA tile kernel
DP4A_MAX_B = 1


# split-K scratch of the tile-packed GEMV, one per device: partial sums and per-tile tickets.
# Launches on one stream reuse it in turn; the kernel leaves the tickets at zero.
_TG_PART_FLOATS = 1 << 21
_TG_TICKETS = 1 << 16
_tg_ws: dict = {}


def tgemv_workspace(device, weights=()) -> tuple[torch.Tensor, torch.Tensor]:
    """Split-K scratch sized for every matrix in ``weights`` (QuantWeights with a tile-packed copy).
    Allocate before any CUDA-graph capture: its addresses are baked into graphs."""
    key = torch.device(device)
    need_p, need_t = _TG_PART_FLOATS, _TG_TICKETS
    for w in weights:
        if w is not None and w.tp is not None:
            p, t = ext().tgemv_workspace(w.qtype, w.rows, w.cols, key.index or 0)[:2]
            need_p, need_t = max(need_p, p), max(need_t, t)
    ws = _tg_ws.get(key)
    if ws is None or ws[0].numel() < need_p or ws[1].numel() < need_t:
        ws = (torch.zeros(need_p, dtype=torch.float32, device=key), torch.zeros(need_t, dtype=torch.int32, device=key))
        _tg_ws[key] = ws
    return ws


def gemv(w, act: ActQ, B: int, y: torch.Tensor, bias: torch.Tensor | None = None, epi: int = EPI_STORE,
         flags: int = 0, ar: tuple | None = None, prefetch: torch.Tensor | None = None) -> None:
    """y[:B] (op)= W . x for a decode batch (w: models.weights.QuantWeight); chunks of 8 tokens.

    Matrices with a tile-packed copy (``QuantWeight.pack``) run the tile-packed tensor-core GEMV;
    others the row-major kernels.  ``ar`` = (peer bases, rank, line-slot offset, epochs [, spin
    limit]) fuses a tensor-parallel all-reduce of the result into the GEMV (EPI_ADD, one
    launch, B <= 32); a peer that never arrives makes the wait give up after the spin limit (0: the
    kernel default) and report error 4 in the registered error word."""
    C = ext()
    if w.tp is not None:
        part, cnt = tgemv_workspace(w.tp.device)
        need = getattr(w, "_tg_need", None)
        if need is None:
            need = w._tg_need = tuple(ext().tgemv_workspace(w.qtype, w.rows, w.cols, w.tp.device.index or 0)[:2])
        if part.numel() < need[0] or cnt.numel() < need[1]:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("tgemv scratch too small inside a graph capture: size it beforehand "
                                   "(ops.kernels.tgemv_workspace(device, weights))")
            part, cnt = tgemv_workspace(w.tp.device, (w,))
        for b0 in range(0, B, TGEMV_MAX_B):
            nb = min(TGEMV_MAX_B, B - b0)
            if ar is not None and B > TGEMV_MAX_B:
                raise ValueError("the fused all-reduce GEMV takes at most 32 tokens")
            arkw = {} if ar is None else dict(ar_peers=ar[0], ar_me=ar[1], ar_parts_off=ar[2], ar_epochs=ar[3],
                                              ar_spin_limit=ar[4] if len(ar) > 4 else 0)
            if prefetch is not None and b0 == 0:
                arkw["prefetch"] = prefetch
            ew = _err_word.get(w.tp.device)
            if isinstance(act, FAct):
                C.tgemv(w.tp, w.qtype, w.rows, w.cols, None, None, act.x[b0:b0 + nb], act.gamma, act.eps, nb,
                        y[b0:b0 + nb], bias, epi, part, cnt, ew, flags, **arkw)
            else:
                C.tgemv(w.tp, w.qtype, w.rows, w.cols, act.q[b0:b0 + nb], act.ds[b0:b0 + nb], None, None, 0.0, nb,
                        y[b0:b0 + nb], bias, epi, part, cnt, ew, flags, unit=getattr(act, "unit", False), **arkw)
            count()
        return
    if isinstance(act, FAct):
        raise RuntimeError("fp32 activations need the tile-packed weights (QuantWeight.pack)")
    for b0 in range(0, B, GEMV_MAX_B):
        nb = min(GEMV_MAX_B, B - b0)
        q = act.q[b0:b0 + nb]
        d = act.ds[b0:b0 + nb]
        if nb <= DP4A_MAX_B and epi != EPI_SWIGLU:
            C.qgemv(w.buf, w.qtype, w.rows, w.cols, w.pitch, q, d, nb, y[b0:b0 + nb], bias, epi)
        else:
            C.qmmv(w.buf, w.qtype, w.rows, w.cols, w.pitch, q, d, nb, y[b0:b0 + nb], bias, epi)
        count()


_pair_plans: dict = {}


def gemv_pair(wa, wb, act: ActQ, B: int, ya: torch.Tensor, yb: torch.Tensor, bias_a: torch.Tensor | None = None,
              bias_b: torch.Tensor | None = None, prefetch: torch.Tensor | None = None) -> bool:
    """ya[:B] = Wa . x (+ bias_a) and yb[:B] = Wb . x (+ bias_b) in ONE launch of the tile-packed GEMV
    (two matrices of different block formats over the same quantized activations, e.g. q|k in Q4_K
    and v in Q6_K): the SMs are shared in proportion to the weight bytes, so the two launches' latency
    chains overlap.  Returns False (nothing launched) when the pair has no such launch; the caller
    then runs the two GEMVs one after the other."""
    if wa.tp is None or wb.tp is None or isinstance(act, FAct) or wa.cols != wb.cols:
        return False
    if (wa.qtype, wb.qtype) == (14, 12):   # the launch takes the Q4_K matrix first
        wa, wb, ya, yb, bias_a, bias_b = wb, wa, yb, ya, bias_b, bias_a
    dev = wa.tp.device
    chunks = [(b0, min(TGEMV_MAX_B, B - b0)) for b0 in range(0, B, TGEMV_MAX_B)]
    for _, nb in chunks:
        key = (wa.qtype, wa.rows, wb.qtype, wb.rows, wa.cols, nb, dev)
        plan = _pair_plans.get(key)
        if plan is None:
            plan = _pair_plans[key] = tuple(ext().tgemv_pair_plan(wa.qtype, wa.rows, wb.qtype, wb.rows, wa.cols, nb,
                                                                  dev.index or 0))
        if not plan:
            return False
        part, cnt = tgemv_workspace(dev)
        if part.numel() < plan[1] or cnt.numel() < plan[2]:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("tgemv scratch too small for a pair launch inside a graph capture")
            return False
    for b0, nb in chunks:
        ext().tgemv_pair(wa.tp, wa.qtype, wa.rows, ya[b0:b0 + nb], bias_a, wb.tp, wb.qtype, wb.rows, yb[b0:b0 + nb],
                         bias_b, wa.cols, act.q[b0:b0 + nb], act.ds[b0:b0 + nb], nb, part, cnt, _err_word.get(dev),
                         prefetch if b0 == 0 else None, getattr(act, "unit", False))
        count()
    return True


def decode_attention(q, k_cache, v_cache, block_table, ctx_len, n_split: int, out=None, act: ActQ | None = None,
                     workspace=None, ldo: int = 0, tickets=None, prefetch: torch.Tensor | None = None,
                     window: int = 0, shared_pages: torch.Tensor | None = None, prefix_splits: int = 0,
                     scale: float = 0.0, softcap: float = 0.0, pages_per_split: int = 1,
                     sinks: torch.Tensor | None = None) -> None:
    """n_split splits of at least pages_per_split pages each (a sequence's live pages spread evenly
    over the splits when there are more; splits past its pages are skipped).
    ldo: elements per token row of the output (default: heads x head_dim).  tickets: zeroed int32
    [B * kv heads]; when given, the last split of each (sequence, KV group) merges the splits in the
    same kernel instead of a separate combine launch (the kernel leaves the tickets at zero).
    window > 0: sliding-window attention over the last ``window`` keys.
    shared_pages (int32 [1] on the device) with prefix_splits > 0: cascade attention -- the first
    *shared_pages pages, identical in every block table, are attended once for the whole batch
    (workspace sized for n_split + prefix_splits slots)."""
    ext().decode_attention(q, k_cache, v_cache, block_table, ctx_len, n_split, pages_per_split, out,
                           act.q if act is not None else None, act.ds if act is not None else None, workspace, ldo,
                           tickets, prefetch, window, shared_pages, prefix_splits, scale, softcap, sinks)
    cascade = shared_pages is not None and prefix_splits > 0 and window <= 0 and \
        q.shape[0] * (q.shape[1] // k_cache.shape[1]) <= 64
    n_slots = n_split + (prefix_splits if cascade else 0)
    count((1 if cascade else 0) + (2 if n_slots > 1 and (tickets is None or cascade) else 1))


def prefill_attention(q, k_cache, v_cache, block_table, meta, out, window: int = 0, scale: float = 0.0,
                      softcap: float = 0.0, sinks: torch.Tensor | None = None) -> None:
    """scale: logit scale (0 = 1/sqrt(head_dim)); softcap > 0: logits cap * tanh(logit / cap);
    sinks [H] f32: one extra softmax logit per head that attends to nothing (gpt-oss)."""
    ext().prefill_attention(q, k_cache, v_cache, block_table, meta.tile_seq, meta.tile_q0, meta.seq_qoff,
                            meta.seq_qlen, meta.seq_pos0, meta.n_tiles, out, window, scale, softcap, sinks)
    count()


def prefill_attention_tc(q, k_cache_all, v_cache_all, layer: int, block_table, meta, out, err=None) -> None:
    """Causal paged prefill attention on tcgen05 / TMEM: q [T, H, 128] bf16, the whole caches
    [L, P, Hkv, 16, 128] and the layer index (one TMA map covers every layer), out [T, H*128] bf16."""
    ext().prefill_attention_tc(q, k_cache_all, v_cache_all, layer, block_table, meta.tile128_seq, meta.tile128_q0,
                               meta.seq_qoff, meta.seq_qlen, meta.seq_pos0, meta.n_tiles128, out, err)
    count()


def kv_move(kv, src_slot: torch.Tensor, dst_slot: torch.Tensor, rot: torch.Tensor, cos_n: torch.Tensor,
            sin_n: torch.Tensor) -> None:
    """Move K/V rows (all layers) from src to dst slots; keys of rows with rot=1 are re-rotated back
    by the shift whose cos/sin per pair are cos_n / sin_n."""
    ext().kv_move(kv.k, kv.v, src_slot, dst_slot, rot, cos_n, sin_n)
    count()


def embed(w, ids: torch.Tensor, out_f32=None, out_bf16=None, err=None, scale: float = 1.0) -> None:
    ext().embed(w.buf, w.qtype, w.pitch, w.rows, w.cols, ids, out_f32, out_bf16, err, scale)
    count()


def rmsnorm_add(y: torch.Tensor, w: torch.Tensor, eps: float, x: torch.Tensor) -> None:
    """x += rmsnorm(y) * w (row-wise; sandwich norms before the residual add)."""
    ext().rmsnorm_add(y, w, eps, x)
    count()


def rope_kv(qkv, pos, slot, cos, sin, H, Hkv, q_norm, k_norm, eps, q_f32, q_bf16, k_cache, v_cache) -> None:
    ext().rope_kv(qkv, pos, slot, cos, sin, H, Hkv, q_norm, k_norm, eps, q_f32, q_bf16, k_cache, v_cache)
    count()


def rmsnorm_bf16(x, w, eps, y) -> None:
    ext().rmsnorm_bf16(x, w, eps, y)
    count()


_argmax_ws: dict = {}


def argmax_workspace(device, rows: int = 256) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-device scratch of the multi-CTA argmax (packed keys, tickets; left at zero by every
    launch).  Allocate it before any CUDA-graph capture: its addresses are baked into graphs."""
    key = torch.device(device)
    ws = _argmax_ws.get(key)
    if ws is None or ws[0].numel() < rows:
        n = max(rows, 256)
        ws = (torch.zeros(n, dtype=torch.int64, device=key), torch.zeros(n, dtype=torch.int32, device=key))
        _argmax_ws[key] = ws
    return ws


def argmax(logits: torch.Tensor, V: int, out: torch.Tensor) -> None:
    """First-index argmax of each row over the first V columns."""
    keys, tickets = argmax_workspace(logits.device, logits.shape[0])
    ext().argmax_rows(logits, V, out, keys, tickets)
    count()


def gemm(a: torch.Tensor, w, out: torch.Tensor, epi: int = EPI_STORE, bias: torch.Tensor | None = None,
         err: torch.Tensor | None = None) -> None:
    """out (op)= a[M,K] (bf16) . W^T on the tcgen05 tensor cores (W: QuantWeight -> its dense bf16 copy)."""
    ext().gemm_bf16(a, w.dense() if not isinstance(w, torch.Tensor) else w, out, bias, epi, err)
    count()
