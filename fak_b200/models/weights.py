"""Device-resident model weights.

Quantized matrices keep their GGML block bytes unchanged; rows are placed at a 16-byte
pitch (``ops.quant.row_pitch``) so every row starts on a 16-byte boundary for wide and
asynchronous loads.  Row permutations are exact on quantized rows, which the loader uses to

* fuse q/k/v into one matrix when their block types match (one GEMV launch);
* interleave gate/up rows in blocks of 8 (``interleave_gate_up``) so the GEMV/GEMM epilogues
  can apply SwiGLU without a second pass (reference fused-op boundary: SwiGLUMatMulAddInPlace,
  internal/model/hal.go:204-255);
* restore HF rotary row order for GGML "llama" checkpoints (done in ``models.loader``).

Float checkpoints (f32/f16/bf16 matrices) are quantized to Q8_0 on load, as the reference's
quant-on-load path does (internal/ggufload/gguf_weightsource.go:35-60).

Tensor parallel sharding happens here too (``shard`` describes this rank's slice); the
plan itself lives in ``parallel.tp``.
"""
from __future__ import annotations

import dataclasses
import os
import warnings
from typing import Callable, Iterator

import numpy as np
import torch

from ..config import ModelConfig
from ..gguf import GGMLType
from ..gguf.quants import quantize as np_quantize, dequantize as np_dequantize
from ..ops import quant as dq


@dataclasses.dataclass
class QuantWeight:
    """A [rows, cols] matrix of GGML blocks on the device at a 16-byte row pitch."""
    buf: torch.Tensor  # uint8, rows * pitch (+ slack)
    qtype: int
    rows: int
    cols: int
    pitch: int
    _dense: torch.Tensor | None = None
    tp: torch.Tensor | None = None  # tile-packed copy for the decode GEMV (``ops.quant.tile_pack``)

    @classmethod
    def from_rows(cls, rows_u8: torch.Tensor, qtype: int, cols: int, device: torch.device) -> "QuantWeight":
        rows = int(rows_u8.shape[0])
        packed = dq.row_bytes(qtype, cols)
        if rows_u8.shape[1] != packed:
            raise ValueError(f"row bytes {rows_u8.shape[1]} != expected {packed} for {GGMLType(qtype).name}x{cols}")
        pitch = dq.row_pitch(qtype, cols)
        # slack: tile copies may read up to one pitch past the last row
        buf = torch.zeros(rows * pitch + pitch + 256, dtype=torch.uint8, device=device)
        src = rows_u8.to(device, non_blocking=False)
        buf[: rows * pitch].view(rows, pitch)[:, :packed].copy_(src)
        return cls(buf, int(qtype), rows, int(cols), pitch)

    def dense(self, dtype: torch.dtype = torch.bfloat16, cache: bool = True) -> torch.Tensor:
        """Dequantized [rows, cols] copy (used by the prefill GEMMs); cached when requested."""
        if self._dense is not None and self._dense.dtype == dtype:
            return self._dense
        d = dq.dequantize_rows(self.buf, self.qtype, self.rows, self.cols, self.pitch, dtype)
        if cache:
            self._dense = d
        return d

    def pack(self) -> "QuantWeight":
        """Build the tile-packed copy the decode GEMV reads (Q4_K / Q6_K / Q8_0 matrices)."""
        if self.tp is None and self.qtype in dq.TILE_UNIT_BYTES and self.buf.is_cuda:
            self.tp = dq.tile_pack(self.buf, self.qtype, self.rows, self.cols, self.pitch)
        return self

    @property
    def nbytes(self) -> int:
        return self.rows * dq.row_bytes(self.qtype, self.cols)


@dataclasses.dataclass
class LayerWeights:
    attn_norm: torch.Tensor
    ffn_norm: torch.Tensor
    qkv: list[tuple[QuantWeight, int]]   # (segment, first output column)
    qkv_bias: torch.Tensor | None
    q_norm: torch.Tensor | None
    k_norm: torch.Tensor | None
    o: QuantWeight
    gate_up: QuantWeight | None          # interleaved rows (dense FFN)
    down: QuantWeight | None
    router: torch.Tensor | None = None   # [E, d] f32 (MoE)
    experts_gate_up: QuantWeight | None = None  # local experts stacked, 8-row interleaved gate/up
    experts_down: QuantWeight | None = None
    expert_ids: list[int] | None = None  # global ids of the experts held here
    post_attn_norm: torch.Tensor | None = None   # sandwich norms (Gemma-2): after o_proj / down
    post_ffn_norm: torch.Tensor | None = None
    # gpt-oss: attention sinks of this rank's heads [Hq_local], the o_proj bias [d], the router bias
    # [E], and per-expert biases of the local experts (gate/up rows interleaved as the weights)
    attn_sinks: torch.Tensor | None = None
    o_bias: torch.Tensor | None = None
    router_bias: torch.Tensor | None = None
    experts_gate_up_bias: torch.Tensor | None = None
    experts_down_bias: torch.Tensor | None = None


@dataclasses.dataclass
class ModelWeights:
    cfg: ModelConfig
    embed: QuantWeight
    layers: list[LayerWeights]
    final_norm: torch.Tensor
    lm_head: QuantWeight
    q_heads: list[int]        # global q-head ids on this rank
    kv_heads: list[int]       # global kv-head ids on this rank
    ffn_slice: tuple[int, int]  # [start, end) of the FFN dim on this rank
    tp_rank: int = 0
    tp_size: int = 1
    load_profile: dict = dataclasses.field(default_factory=dict)   # seconds per load phase
    # o_proj input columns: this rank holds columns [a0, a1) of the attention output projection; its
    # own heads' outputs fill [c0, c1) and the rest of [a0, a1) stays zero (a1 - a0 == the matrix's K)
    o_cols: tuple[int, int, int, int] = (0, 0, 0, 0)

    @property
    def n_q_local(self) -> int:
        return len(self.q_heads)

    @property
    def n_kv_local(self) -> int:
        return len(self.kv_heads)

    def nbytes(self) -> int:
        n = self.embed.nbytes + self.lm_head.nbytes
        for L in self.layers:
            n += sum(s.nbytes for s, _ in L.qkv) + L.o.nbytes
            if L.gate_up is not None:
                n += L.gate_up.nbytes + L.down.nbytes
            if L.experts_gate_up is not None:
                n += L.experts_gate_up.nbytes + L.experts_down.nbytes
        return n


# ------------------------------------------------------------------------------------------
# raw tensor sources: a GGUF file, or tensors synthesized directly on the device
# ------------------------------------------------------------------------------------------
RawGetter = Callable[[str], tuple[tuple[int, ...], int, torch.Tensor]]  # -> (shape, ggml type, uint8 rows)


def gguf_source(path: str) -> tuple[ModelConfig, RawGetter, Callable[[], None]]:
    from .loader import llama_rope_unpermute_rows, open_model
    g, cfg = open_model(path)

    def get(name: str):
        ti = g.tensors[name]
        raw = g.raw_rows(name) if len(ti.shape) >= 2 else g.raw(name).reshape(1, -1)
        if cfg.arch == "llama" and (name.endswith("attn_q.weight") or name.endswith("attn_k.weight")):
            heads = cfg.n_heads if name.endswith("attn_q.weight") else cfg.n_kv_heads
            raw = llama_rope_unpermute_rows(raw, heads, cfg.head_dim)
        with warnings.catch_warnings():   # read-only memory map: the rows are only read
            warnings.simplefilter("ignore", UserWarning)
            return ti.shape, int(ti.ggml_type), torch.from_numpy(np.ascontiguousarray(raw))

    return cfg, get, g.close


def synthetic_source(cfg: ModelConfig, mix: str = "q4_k_m", seed: int = 0, std: float = 0.02,
                     device: str = "cuda") -> tuple[ModelConfig, RawGetter, Callable[[], None]]:
    """Weights generated and block-quantized on the GPU (no file): same types as the GGUF writer."""
    from ..gguf.synth import _seed_for, choose_type, tensor_plan
    plan = {name: (shape, role) for name, shape, role in tensor_plan(cfg)}

    def get(name: str):
        shape, role = plan[name]
        t = int(choose_type(cfg, name, shape, role, mix))
        raw = dq.synth_quantized(shape, t, _seed_for(seed, name), std, ones=(role == "norm"), device=device)
        rows = raw.view(int(np.prod(shape[:-1])) if len(shape) > 1 else 1, -1)
        return shape, t, rows

    return cfg, get, lambda: None


# ------------------------------------------------------------------------------------------
# loading
# ------------------------------------------------------------------------------------------
def _vec(get: RawGetter, name: str, device) -> torch.Tensor:
    shape, t, raw = get(name)
    arr = raw.cpu().numpy().reshape(-1) if raw.is_cuda else raw.numpy().reshape(-1)
    return torch.from_numpy(np_dequantize(arr, t).astype(np.float32)).to(device)


def _as_device_quant(shape, t: int, raw: torch.Tensor, device) -> tuple[torch.Tensor, int]:
    """Rows of a supported device block type; float matrices are quantized to Q8_0 on load."""
    if t in dq.DEVICE_QTYPES:
        return raw.view(torch.uint8), t
    cols = shape[-1]
    if raw.is_cuda:
        x = raw.view({GGMLType.F32: torch.float32, GGMLType.F16: torch.float16,
                      GGMLType.BF16: torch.bfloat16}[GGMLType(t)]).float()
        q = dq.quantize_blocks(x.reshape(-1), dq.QT_Q8_0)
    else:
        f = np_dequantize(raw.numpy().reshape(-1), t)
        q = torch.from_numpy(np_quantize(f, GGMLType.Q8_0))
    return q.view(-1, dq.row_bytes(dq.QT_Q8_0, cols)), dq.QT_Q8_0


def head_assignment(cfg: ModelConfig, tp_rank: int, tp_size: int) -> tuple[list[int], list[int]]:
    """(q heads, kv heads) owned by a TP rank.

    Heads are dealt out contiguously.  When there are fewer KV heads than ranks, each KV head
    is replicated on tp_size / n_kv ranks and its query group is split between them as evenly
    as possible (e.g. Qwen2.5-7B at TP=8: 4 KV heads, 7 q-heads per group -> 4 + 3).
    """
    H, Hk, T = cfg.n_heads, cfg.n_kv_heads, tp_size
    G = H // Hk
    if T == 1:
        return list(range(H)), list(range(Hk))
    if Hk >= T:
        if Hk % T:
            raise ValueError(f"{Hk} KV heads cannot be split over {T} ranks")
        per = Hk // T
        kv = list(range(tp_rank * per, (tp_rank + 1) * per))
        return [h for k in kv for h in range(k * G, (k + 1) * G)], kv
    if T % Hk:
        raise ValueError(f"TP={T} must be a multiple of the {Hk} KV heads when it exceeds them")
    R = T // Hk
    k = tp_rank // R
    sub = tp_rank % R
    if G < R:
        raise ValueError(f"query group of {G} heads cannot be split over {R} ranks")
    base, extra = divmod(G, R)
    start = sub * base + min(sub, extra)
    n = base + (1 if sub < extra else 0)
    return [k * G + start + i for i in range(n)], [k]


def o_proj_columns(cfg: ModelConfig, q_heads: list[int], tp_size: int) -> tuple[int, int, int, int]:
    """(a0, a1, c0, c1): the row-parallel slice of the attention output projection a rank holds.

    The rank's heads produce input columns [c0, c1) = [first head * D, (last head + 1) * D).  Quantized
    rows can only be cut on block boundaries (256 weights for K-quant super-blocks and the int4 group
    format; 64 suffices for Q8_0 in the tile-packed GEMV and is used when the width is not a multiple
    of 256, which K-quant rows never are), so the rank keeps the aligned range [a0, a1) around
    its heads and feeds zero activations (zero codes and zero block scales) to the columns of other
    ranks' heads inside it: those weights then contribute exactly zero, and the rank-order sum of the
    partial outputs over ranks is the full projection.  Qwen2.5-7B at TP=8 (3 or 4 heads of 128 per
    rank) keeps 512 or 768 of the 3584 columns instead of the whole matrix."""
    K = cfg.n_heads * cfg.head_dim
    if tp_size == 1:
        return 0, K, 0, K
    D = cfg.head_dim
    c0, c1 = q_heads[0] * D, (q_heads[-1] + 1) * D
    if q_heads != list(range(q_heads[0], q_heads[-1] + 1)):
        raise ValueError("row-parallel o_proj expects each rank's query heads to be contiguous")
    g = 256 if K % 256 == 0 else 64   # one slice for every layer, whatever its block type
    a0 = c0 // g * g
    a1 = min(K, -(-c1 // g) * g)
    return a0, a1, c0, c1


def vocab_slice(V: int, tp_rank: int, tp_size: int) -> tuple[int, int]:
    per = -(-V // tp_size)
    return min(V, tp_rank * per), min(V, (tp_rank + 1) * per)


def ffn_assignment(ffn: int, tp_rank: int, tp_size: int, granule: int) -> tuple[int, int]:
    """[start, end) of the FFN dim on a rank, in whole ``granule`` units (a K-quant super-block)."""
    units = ffn // granule
    base, extra = divmod(units, tp_size)
    start = tp_rank * base + min(tp_rank, extra)
    n = base + (1 if tp_rank < extra else 0)
    return start * granule, (start + n) * granule


def interleave_gate_up(g_rows: torch.Tensor, u_rows: torch.Tensor, block: int = 8) -> torch.Tensor:
    """Rows [16i, 16i+8) = gate rows [8i, 8i+8), rows [16i+8, 16i+16) = up rows [8i, 8i+8).

    The GEMV and GEMM SwiGLU epilogues rely on this layout: a 16-row MMA tile (or a
    16-column accumulator chunk) then holds matching gate and up values in the same thread.
    """
    n = g_rows.shape[0]
    if n % block or u_rows.shape[0] != n:
        raise ValueError(f"gate/up rows ({n}) must be a multiple of {block}")
    g = g_rows.reshape(n // block, block, -1)
    u = u_rows.reshape(n // block, block, -1)
    return torch.stack([g, u], dim=1).reshape(2 * n, -1)


def _rows_of(raw: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
    return raw.index_select(0, idx.to(raw.device))


def _col_block_slice(raw: torch.Tensor, t: int, cols: int, c0: int, c1: int) -> torch.Tensor:
    """Columns [c0, c1) of quantized rows, on block boundaries."""
    from ..gguf.constants import BLOCK_INFO
    blk, nb = BLOCK_INFO[GGMLType(t)]
    if c0 % blk or c1 % blk:
        raise ValueError(f"column slice [{c0},{c1}) not on {blk}-element block boundaries")
    return raw[:, c0 // blk * nb: c1 // blk * nb].contiguous()


def load_weights(source: tuple[ModelConfig, RawGetter, Callable[[], None]], device: str | torch.device = "cuda",
                 tp_rank: int = 0, tp_size: int = 1, expert_filter: tuple[int, int] | None = None,
                 prefill_dense: bool = False, repeat_layers: bool = False,
                 offload_experts: bool = False) -> ModelWeights:
    """repeat_layers: load only block 0 and let every layer share it (smoke tests of a large
    architecture: the same shapes and kernels, one layer's worth of weight synthesis and memory).
    offload_experts: MoE expert matrices stay in host memory in their GGML blocks (their FFNs run
    on the CPU, ``models.moe_offload``); a layer's experts pass through the device only while it
    is converted."""
    import time
    cfg, get0, close = source
    device = torch.device(device)
    prof = {"read": 0.0, "convert": 0.0, "pack": 0.0, "dense": 0.0}
    t_start = time.perf_counter()

    def get(name: str):   # tensor reads, timed for the load profile
        t = time.perf_counter()
        try:
            return get0(name)
        finally:
            prof["read"] += time.perf_counter() - t
    D = cfg.head_dim
    q_heads, kv_heads = head_assignment(cfg, tp_rank, tp_size)
    granule = 256
    ffn_dim = cfg.expert_ffn_dim if cfg.is_moe else cfg.ffn_dim
    if ffn_dim % granule:
        granule = 32 if ffn_dim % 32 == 0 else ffn_dim
    f0, f1 = ffn_assignment(ffn_dim, tp_rank, tp_size, granule) if not cfg.is_moe else (0, ffn_dim)

    def quant(name: str) -> tuple[tuple[int, ...], int, torch.Tensor]:
        shape, t, raw = get(name)
        t0 = time.perf_counter()
        rows2, t2 = _as_device_quant(shape, t, raw, device)
        prof["convert"] += time.perf_counter() - t0
        return shape, t2, rows2

    emb_shape, emb_t, emb_raw = get("token_embd.weight")
    if emb_t == int(GGMLType.G4):   # the embedding gather reads K-quant / Q8_0 / float rows
        emb_raw, emb_t = _as_device_quant(emb_shape, int(GGMLType.F32), torch.from_numpy(
            np_dequantize(emb_raw.cpu().numpy().reshape(-1), emb_t).astype(np.float32)).view(torch.uint8), device)
        emb_raw = emb_raw.cpu()
    if emb_t in (int(GGMLType.F32), int(GGMLType.F16), int(GGMLType.BF16)) or emb_t in dq.DEVICE_QTYPES:
        embed = QuantWeight.from_rows(emb_raw.view(torch.uint8).reshape(emb_shape[0], -1), emb_t, emb_shape[1], device)
    else:
        raise ValueError(f"embedding type {GGMLType(emb_t).name} unsupported on the device")

    def head_rows(heads: list[int]) -> torch.Tensor:
        return torch.cat([torch.arange(h * D, (h + 1) * D) for h in heads]) if heads else torch.zeros(0, dtype=torch.long)

    layers = []
    for i in range(1 if repeat_layers else cfg.n_layers):
        p = f"blk.{i}."
        segs: list[tuple[QuantWeight, int]] = []
        parts = []
        for nm, heads in (("attn_q", q_heads), ("attn_k", kv_heads), ("attn_v", kv_heads)):
            shape, t, raw = quant(p + nm + ".weight")
            parts.append((t, _rows_of(raw, head_rows(heads))))
        # merge adjacent segments of the same type into one matrix
        off = 0
        cur_t, cur_rows, cur_off = None, [], 0
        for t, rows in parts:
            if cur_t is not None and t != cur_t:
                segs.append((QuantWeight.from_rows(torch.cat(cur_rows), cur_t, cfg.d_model, device), cur_off))
                cur_rows, cur_off = [], off
            cur_t = t
            cur_rows.append(rows)
            off += rows.shape[0]
        segs.append((QuantWeight.from_rows(torch.cat(cur_rows), cur_t, cfg.d_model, device), cur_off))
        bias = None
        if cfg.qkv_bias:
            qb = _vec(get, p + "attn_q.bias", device)[head_rows(q_heads).to(device)]
            kb = _vec(get, p + "attn_k.bias", device)[head_rows(kv_heads).to(device)]
            vb = _vec(get, p + "attn_v.bias", device)[head_rows(kv_heads).to(device)]
            bias = torch.cat([qb, kb, vb]).contiguous()
        qn = _vec(get, p + "attn_q_norm.weight", device) if cfg.qk_norm else None
        kn = _vec(get, p + "attn_k_norm.weight", device) if cfg.qk_norm else None
        # o_proj is row-parallel (split along its input): each rank multiplies its own heads'
        # outputs into a partial of the full output row, and the partials are summed across ranks
        # (in the GEMV epilogue on the fused path); see o_proj_columns for the block-aligned slice.
        shape, t, raw = quant(p + "attn_output.weight")
        o_cols = o_proj_columns(cfg, q_heads, tp_size)
        if (o_cols[0], o_cols[1]) != (0, shape[1]):
            raw = _col_block_slice(raw, t, shape[1], o_cols[0], o_cols[1])
        o = QuantWeight.from_rows(raw, t, o_cols[1] - o_cols[0], device)
        L = LayerWeights(
            attn_norm=_vec(get, p + "attn_norm.weight", device),
            ffn_norm=_vec(get, p + "ffn_norm.weight", device),
            qkv=segs, qkv_bias=bias, q_norm=qn, k_norm=kn, o=o, gate_up=None, down=None,
        )
        if cfg.sandwich_norms:
            L.post_attn_norm = _vec(get, p + "post_attention_norm.weight", device)
            L.post_ffn_norm = _vec(get, p + "post_ffw_norm.weight", device)
        if cfg.attn_sinks:
            L.attn_sinks = _vec(get, p + "attn_sinks.weight", device)[torch.tensor(q_heads, device=device)].contiguous()
        if cfg.attn_out_bias:
            L.o_bias = _vec(get, p + "attn_output.bias", device)
        if cfg.is_moe:
            # expert parallelism rides on the tensor-parallel group: rank r owns a band of experts
            band = expert_filter if expert_filter is not None else expert_slice(cfg.n_experts, tp_rank, tp_size)
            _load_moe_layer(cfg, get, quant, p, L, device, band, offload_experts)
        else:
            gs, gt, graw = quant(p + "ffn_gate.weight")
            us, ut, uraw = quant(p + "ffn_up.weight")
            if gt != ut:
                raise ValueError(f"layer {i}: gate ({gt}) and up ({ut}) block types differ")
            inter = interleave_gate_up(graw[f0:f1], uraw[f0:f1])
            L.gate_up = QuantWeight.from_rows(inter, gt, cfg.d_model, device)
            ds_, dt, draw = quant(p + "ffn_down.weight")
            if tp_size > 1:
                draw = _col_block_slice(draw, dt, ds_[1], f0, f1)
            L.down = QuantWeight.from_rows(draw, dt, f1 - f0, device)
        t0 = time.perf_counter()
        for s, _ in L.qkv:
            s.pack()
        L.o.pack()
        if L.gate_up is not None:
            L.gate_up.pack()
            L.down.pack()
        t1 = time.perf_counter()
        if prefill_dense:
            for s, _ in L.qkv:
                s.dense()
            L.o.dense()
            if L.gate_up is not None:
                L.gate_up.dense()
                L.down.dense()
        prof["pack"] += t1 - t0
        prof["dense"] += time.perf_counter() - t1
        layers.append(L)
    if repeat_layers:
        layers = layers * cfg.n_layers
    final_norm = _vec(get, "output_norm.weight", device)
    # lm_head: split by vocab rows under TP (ceil(V/T) rows per rank, the last rank may hold fewer)
    v0, v1 = vocab_slice(cfg.vocab_size, tp_rank, tp_size)
    if cfg.tie_embeddings and tp_size == 1 and emb_t in dq.DEVICE_QTYPES:
        lm_head = embed
    else:
        shape, t, raw = quant("token_embd.weight" if cfg.tie_embeddings else "output.weight")
        lm_head = QuantWeight.from_rows(raw[v0:v1].contiguous(), t, shape[1], device)
    lm_head.pack()
    close()
    if device.type == "cuda":
        torch.cuda.synchronize(device)
    prof["total"] = time.perf_counter() - t_start
    prof["upload"] = max(0.0, prof["total"] - prof["read"] - prof["convert"] - prof["pack"] - prof["dense"])
    return ModelWeights(cfg, embed, layers, final_norm, lm_head, q_heads, kv_heads, (f0, f1), tp_rank, tp_size,
                        load_profile={k: round(v, 4) for k, v in prof.items()}, o_cols=o_cols)


def expert_slice(E: int, rank: int, size: int) -> tuple[int, int]:
    """Contiguous band of experts owned by an expert-parallel rank (reference: ExpertParallelPlan,
    internal/model/expert_parallel.go:68-83)."""
    per = -(-E // size)
    return min(E, rank * per), min(E, (rank + 1) * per)


def _load_moe_layer(cfg, get, quant, p, L: LayerWeights, device, expert_filter, offload: bool = False) -> None:
    E, f, d = cfg.n_experts, cfg.expert_ffn_dim, cfg.d_model
    L.router = _vec(get, p + "ffn_gate_inp.weight", device).view(E, d).contiguous()
    e0, e1 = expert_filter if expert_filter is not None else (0, E)
    gs, gt, graw = quant(p + "ffn_gate_exps.weight")
    us, ut, uraw = quant(p + "ffn_up_exps.weight")
    ds_, dt, draw = quant(p + "ffn_down_exps.weight")
    graw = graw.view(E, f, -1)
    uraw = uraw.view(E, f, -1)
    draw = draw.view(E, d, -1)
    # experts stored back to back in one buffer (rows of expert e start at e * rows_per_expert)
    gu = torch.cat([interleave_gate_up(graw[e], uraw[e]) for e in range(e0, e1)])
    wdev = torch.device("cpu") if offload else device   # where the expert matrices live
    L.experts_gate_up = QuantWeight.from_rows(gu, gt, d, wdev)
    L.experts_down = QuantWeight.from_rows(draw[e0:e1].reshape((e1 - e0) * d, -1).contiguous(), dt, f, wdev)
    L.expert_ids = list(range(e0, e1))
    if cfg.moe_bias:   # gpt-oss: router and expert biases
        L.router_bias = _vec(get, p + "ffn_gate_inp.bias", device)
        bg = _vec(get, p + "ffn_gate_exps.bias", device).view(E, f)
        bu = _vec(get, p + "ffn_up_exps.bias", device).view(E, f)
        L.experts_gate_up_bias = torch.cat([interleave_gate_up(bg[e][:, None], bu[e][:, None]).view(-1)
                                            for e in range(e0, e1)]).contiguous().to(wdev)
        L.experts_down_bias = _vec(get, p + "ffn_down_exps.bias", device).view(E, d)[e0:e1].reshape(-1) \
            .contiguous().to(wdev)
    if offload:
        return
    if f % 256 == 0 and d % 256 == 0:  # tile-packed copies for the grouped expert GEMV
        L.experts_gate_up.pack()
        L.experts_down.pack()
