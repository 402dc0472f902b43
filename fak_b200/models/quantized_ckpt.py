"""Weight-only int4 checkpoints: AutoAWQ and GPTQ (qweight / qzeros / scales [/ g_idx]) triples.

Both formats store, per linear layer, unsigned codes q, per-(group, output) scales s and zero points
z with w[o, i] = (q[o, i] - z[g(i), o]) * s[g(i), o]:

* AutoAWQ ("gemm" version): qweight int32 [in, out/8] and qzeros int32 [in/g, out/8] packed along the
  OUTPUT dimension, nibble p of each word holding logical column ``AWQ_ORDER[p]`` of its 8; scales
  [in/g, out].
* GPTQ (AutoGPTQ / GPTQModel): qweight int32 [in*bits/32, out] packed along the INPUT dimension
  (sequential, least significant bits first); qzeros int32 [groups, out*bits/32] packed along the
  output dimension; scales [groups, out]; optional g_idx [in] (act-order group of every input).
  Checkpoint format "gptq" (v1) stores zero - 1; "gptq_v2" stores the zero itself.

On the device, 4-bit layers whose groups are contiguous runs of a multiple of 128 inputs become G4
blocks (codes, scale and scale * zero per 128-group; the decode GEMV and prefill dequantizer run
them directly).  Anything else -- act-order g_idx, groups of 32 or 64, 8-bit GPTQ -- is dequantized
to float32 and takes the quant-on-load path like a float checkpoint.

Reference: AWQ group-wise weights (internal/model/awq_group.go), per-channel AWQ (awq.go), GPTQ
(internal/model/gptq.go:3-60, decodeGPTQTensor :304-400).
"""
from __future__ import annotations

import numpy as np

from ..gguf import GGMLType
from ..gguf.quants import G4_GROUP, QK_K, g4_from_codes

AWQ_ORDER = (0, 2, 4, 6, 1, 3, 5, 7)   # logical column held by nibble position p (AutoAWQ packer)


def _nibbles(words: np.ndarray, bits: int) -> np.ndarray:
    """int32 [..., n] -> codes [..., n * 32/bits], least significant field first."""
    w = np.ascontiguousarray(words).view(np.uint32)
    per = 32 // bits
    shifts = (np.arange(per, dtype=np.uint32) * bits)
    out = (w[..., None] >> shifts) & np.uint32((1 << bits) - 1)
    return out.reshape(*w.shape[:-1], w.shape[-1] * per).astype(np.uint8)


def _pack(codes: np.ndarray, bits: int) -> np.ndarray:
    """codes [..., n] (n a multiple of 32/bits) -> int32 [..., n * bits/32]."""
    per = 32 // bits
    c = codes.astype(np.uint32).reshape(*codes.shape[:-1], -1, per)
    shifts = (np.arange(per, dtype=np.uint32) * bits)
    return np.bitwise_or.reduce(c << shifts, axis=-1).astype(np.uint32).view(np.int32)


def _awq_unorder(x: np.ndarray) -> np.ndarray:
    """Position-major nibbles [..., 8k] -> logical column order."""
    n = x.shape[-1]
    inv = np.empty(8, np.int64)
    inv[list(AWQ_ORDER)] = np.arange(8)
    idx = (np.arange(n).reshape(-1, 8)[:, inv]).reshape(-1)
    return x[..., idx]


def _awq_order(x: np.ndarray) -> np.ndarray:
    n = x.shape[-1]
    idx = (np.arange(n).reshape(-1, 8)[:, list(AWQ_ORDER)]).reshape(-1)
    return x[..., idx]


def unpack_awq(qweight: np.ndarray, qzeros: np.ndarray, scales: np.ndarray, group: int):
    """-> codes [out, in] u8, scales [out, groups] f32, zeros [out, groups] f32, group."""
    codes = _awq_unorder(_nibbles(qweight, 4)).T                       # [out, in]
    zeros = _awq_unorder(_nibbles(qzeros, 4)).T.astype(np.float32)     # [out, groups]
    s = np.asarray(scales, np.float32).T
    return np.ascontiguousarray(codes), np.ascontiguousarray(s), np.ascontiguousarray(zeros), group


def pack_awq(codes: np.ndarray, scales: np.ndarray, zeros: np.ndarray):
    """Inverse of ``unpack_awq`` (codes [out, in], scales / zeros [out, groups]) -> AutoAWQ tensors."""
    qweight = _pack(_awq_order(np.ascontiguousarray(codes.T)), 4)
    qzeros = _pack(_awq_order(np.ascontiguousarray(zeros.T.astype(np.uint8))), 4)
    return qweight, qzeros, np.ascontiguousarray(scales.T.astype(np.float16))


def unpack_gptq(qweight: np.ndarray, qzeros: np.ndarray, scales: np.ndarray, g_idx: np.ndarray | None,
                bits: int, group: int, v1: bool = True):
    """-> codes [out, in], scales [out, groups], zeros [out, groups], g_idx [in]."""
    if bits not in (2, 4, 8):
        raise NotImplementedError(f"GPTQ {bits}-bit packing")
    codes = _nibbles(np.ascontiguousarray(qweight.T), bits)            # [out, in]
    zeros = _nibbles(qzeros, bits).astype(np.float32)                  # [groups, out]
    if v1:
        zeros = zeros + 1
    n_in = codes.shape[1]
    gi = np.arange(n_in) // group if g_idx is None else np.asarray(g_idx, np.int64)
    return (np.ascontiguousarray(codes), np.ascontiguousarray(np.asarray(scales, np.float32).T),
            np.ascontiguousarray(zeros.T), gi)


def pack_gptq(codes: np.ndarray, scales: np.ndarray, zeros: np.ndarray, bits: int = 4, v1: bool = True):
    """Inverse of ``unpack_gptq`` for contiguous groups -> (qweight, qzeros, scales f16)."""
    qweight = _pack(np.ascontiguousarray(codes), bits).T.copy()       # [in*bits/32, out]
    z = zeros.T.astype(np.int64) - (1 if v1 else 0)
    qzeros = _pack(np.ascontiguousarray((z & ((1 << bits) - 1)).astype(np.uint8)), bits)
    return qweight, qzeros, np.ascontiguousarray(scales.T.astype(np.float16))


def dequant(codes: np.ndarray, scales: np.ndarray, zeros: np.ndarray, g_idx: np.ndarray) -> np.ndarray:
    g = np.asarray(g_idx, np.int64)
    return ((codes.astype(np.float32) - zeros[:, g]) * scales[:, g]).astype(np.float32)


def device_rows(codes: np.ndarray, scales: np.ndarray, zeros: np.ndarray, g_idx: np.ndarray, group: int,
                bits: int = 4) -> tuple[np.ndarray, int]:
    """(rows, ggml type) for the loaders: G4 blocks when the layout allows, else float32 rows."""
    out_, in_ = codes.shape
    contiguous = np.array_equal(np.asarray(g_idx), np.arange(in_) // group)
    if bits == 4 and contiguous and group % G4_GROUP == 0 and in_ % QK_K == 0:
        return g4_from_codes(codes, scales, zeros, group), int(GGMLType.G4)
    w = dequant(codes, scales, zeros, g_idx)
    return w.view(np.uint8).reshape(out_, -1), int(GGMLType.F32)
