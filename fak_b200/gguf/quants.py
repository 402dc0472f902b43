"""NumPy quantizers and dequantizers for GGML block formats.

These are the host-side (CPU) oracle for the block layouts this framework
keeps resident on the GPU unchanged.  The dequantizers mirror the reference's
per-format decoders (internal/ggufload/gguf_dequant.go:214-836, e.g.
dequantQ4KScalar at :709, dequantQ6KScalar at :803, dequantQ8_0Scalar at :793);
the layouts are fixed by the GGUF format so the bit positions must agree.

The quantizers are this framework's own: a min/max scale search per
sub-block (no iterative refinement).  They produce valid blocks of each
format from float weights, which is what the random-init test and benchmark
checkpoints need.  Every float step is written so that the CUDA quantizer
(csrc/kernels/quant.cu) performs the same IEEE float32 operations in the
same order and therefore produces identical bytes.
"""
from __future__ import annotations

import numpy as np

from .constants import BLOCK_INFO, GGMLType, QK_K

_f16 = np.float16
_f32 = np.float32


def _as_blocks(raw: np.ndarray, nbytes: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw).view(np.uint8).reshape(-1)
    if raw.size % nbytes:
        raise ValueError(f"buffer of {raw.size} bytes is not a whole number of {nbytes}-byte blocks")
    return raw.reshape(-1, nbytes)


def _f16_at(blocks: np.ndarray, off: int) -> np.ndarray:
    return blocks[:, off:off + 2].copy().view(_f16).astype(_f32).reshape(-1)


# ----------------------------------------------------------------------------------------
# Q8_0: [d:f16][qs:int8 x 32]
# ----------------------------------------------------------------------------------------

def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=_f32).reshape(-1, 32)
    amax = np.abs(x).max(axis=1)
    d = (amax / _f32(127.0)).astype(_f16)
    df = d.astype(_f32)
    safe = np.where(df == 0, _f32(1.0), df)
    q = np.rint(x / safe[:, None])
    q = np.where(df[:, None] == 0, 0, q)
    q = np.clip(q, -127, 127).astype(np.int8)
    out = np.empty((x.shape[0], 34), np.uint8)
    out[:, 0:2] = d.view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.reshape(-1)


def dequantize_q8_0(raw: np.ndarray) -> np.ndarray:
    b = _as_blocks(raw, 34)
    d = _f16_at(b, 0)
    q = b[:, 2:].view(np.int8).astype(_f32)
    return (q * d[:, None]).reshape(-1)


# ----------------------------------------------------------------------------------------
# Q4_0 / Q4_1 / Q5_0 / Q5_1 (legacy 32-element blocks; dequant only)
# ----------------------------------------------------------------------------------------

def dequantize_q4_0(raw: np.ndarray) -> np.ndarray:
    b = _as_blocks(raw, 18)
    d = _f16_at(b, 0)
    qs = b[:, 2:18]
    lo = (qs & 0x0F).astype(np.int32) - 8
    hi = (qs >> 4).astype(np.int32) - 8
    q = np.concatenate([lo, hi], axis=1).astype(_f32)
    return (q * d[:, None]).reshape(-1)


def dequantize_q4_1(raw: np.ndarray) -> np.ndarray:
    b = _as_blocks(raw, 20)
    d = _f16_at(b, 0)
    m = _f16_at(b, 2)
    qs = b[:, 4:20]
    q = np.concatenate([qs & 0x0F, qs >> 4], axis=1).astype(_f32)
    return (q * d[:, None] + m[:, None]).reshape(-1)


def _q5_high_bits(qh_bytes: np.ndarray) -> np.ndarray:
    qh = qh_bytes.copy().view(np.uint32).reshape(-1)
    bits = (qh[:, None] >> np.arange(32, dtype=np.uint32)[None, :]) & 1
    return (bits << 4).astype(np.int32)


def dequantize_q5_0(raw: np.ndarray) -> np.ndarray:
    b = _as_blocks(raw, 22)
    d = _f16_at(b, 0)
    hb = _q5_high_bits(b[:, 2:6])
    qs = b[:, 6:22]
    q = np.concatenate([qs & 0x0F, qs >> 4], axis=1).astype(np.int32) | hb
    return ((q - 16).astype(_f32) * d[:, None]).reshape(-1)


def dequantize_q5_1(raw: np.ndarray) -> np.ndarray:
    b = _as_blocks(raw, 24)
    d = _f16_at(b, 0)
    m = _f16_at(b, 2)
    hb = _q5_high_bits(b[:, 4:8])
    qs = b[:, 8:24]
    q = np.concatenate([qs & 0x0F, qs >> 4], axis=1).astype(np.int32) | hb
    return (q.astype(_f32) * d[:, None] + m[:, None]).reshape(-1)


# ----------------------------------------------------------------------------------------
# K-quant 6-bit (scale, min) packing shared by Q4_K and Q5_K: 12 bytes hold 8 pairs.
# byte j (j<4):   sc[j] (6 bits)  | top 2 bits of sc[j+4] in bits 6-7
# byte j+4 (j<4): m[j]  (6 bits)  | top 2 bits of m[j+4]  in bits 6-7
# byte j+8 (j<4): low 4 bits of sc[j+4] | low 4 bits of m[j+4] << 4
# ----------------------------------------------------------------------------------------

def unpack_scale_min_k4(scales: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    s = scales.astype(np.int32)
    sc = np.empty((s.shape[0], 8), np.int32)
    mn = np.empty((s.shape[0], 8), np.int32)
    sc[:, :4] = s[:, 0:4] & 63
    mn[:, :4] = s[:, 4:8] & 63
    sc[:, 4:] = (s[:, 8:12] & 0x0F) | ((s[:, 0:4] >> 6) << 4)
    mn[:, 4:] = (s[:, 8:12] >> 4) | ((s[:, 4:8] >> 6) << 4)
    return sc, mn


def pack_scale_min_k4(sc: np.ndarray, mn: np.ndarray) -> np.ndarray:
    sc = sc.astype(np.int32)
    mn = mn.astype(np.int32)
    out = np.empty((sc.shape[0], 12), np.int32)
    out[:, 0:4] = (sc[:, 0:4] & 63) | ((sc[:, 4:8] >> 4) << 6)
    out[:, 4:8] = (mn[:, 0:4] & 63) | ((mn[:, 4:8] >> 4) << 6)
    out[:, 8:12] = (sc[:, 4:8] & 0x0F) | ((mn[:, 4:8] & 0x0F) << 4)
    return out.astype(np.uint8)


# ----------------------------------------------------------------------------------------
# Q4_K: [d:f16][dmin:f16][scales:12][qs:128] per 256 elements.
# Element c*64 + l (l<32) is the low nibble of qs[c*32+l] (sub-block 2c);
# element c*64 + 32 + l is its high nibble (sub-block 2c+1).  w = d*sc*q - dmin*m.
# ----------------------------------------------------------------------------------------

def quantize_q4_k(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=_f32).reshape(-1, QK_K)
    nb = x.shape[0]
    xs = x.reshape(nb, 8, 32)
    mn = np.minimum(xs.min(axis=2), _f32(0.0))
    mx = xs.max(axis=2)
    scale = (mx - mn) / _f32(15.0)
    mins = -mn
    d = (scale.max(axis=1) / _f32(63.0)).astype(_f16)
    dmin = (mins.max(axis=1) / _f32(63.0)).astype(_f16)
    df = d.astype(_f32)
    dmf = dmin.astype(_f32)
    sc = np.where(df[:, None] > 0, np.rint(scale / np.where(df > 0, df, _f32(1))[:, None]), 0)
    sc = np.clip(sc, 0, 63).astype(np.int32)
    m = np.where(dmf[:, None] > 0, np.rint(mins / np.where(dmf > 0, dmf, _f32(1))[:, None]), 0)
    m = np.clip(m, 0, 63).astype(np.int32)
    eff_s = df[:, None] * sc.astype(_f32)
    eff_m = dmf[:, None] * m.astype(_f32)
    safe = np.where(eff_s > 0, eff_s, _f32(1.0))
    q = np.rint((xs + eff_m[:, :, None]) / safe[:, :, None])
    q = np.where(eff_s[:, :, None] > 0, q, 0)
    q = np.clip(q, 0, 15).astype(np.uint8)  # [nb, 8, 32]
    qs = (q[:, 0::2, :] | (q[:, 1::2, :] << 4)).reshape(nb, 128)
    out = np.empty((nb, 144), np.uint8)
    out[:, 0:2] = d.view(np.uint8).reshape(-1, 2)
    out[:, 2:4] = dmin.view(np.uint8).reshape(-1, 2)
    out[:, 4:16] = pack_scale_min_k4(sc, m)
    out[:, 16:144] = qs
    return out.reshape(-1)


def dequantize_q4_k(raw: np.ndarray) -> np.ndarray:
    b = _as_blocks(raw, 144)
    d = _f16_at(b, 0)
    dmin = _f16_at(b, 2)
    sc, mn = unpack_scale_min_k4(b[:, 4:16])
    qs = b[:, 16:144].reshape(-1, 4, 32)
    q = np.stack([qs & 0x0F, qs >> 4], axis=2).reshape(-1, 8, 32).astype(_f32)
    d1 = d[:, None] * sc.astype(_f32)
    m1 = dmin[:, None] * mn.astype(_f32)
    return (d1[:, :, None] * q - m1[:, :, None]).reshape(-1)


def dequantize_q5_k(raw: np.ndarray) -> np.ndarray:
    b = _as_blocks(raw, 176)
    d = _f16_at(b, 0)
    dmin = _f16_at(b, 2)
    sc, mn = unpack_scale_min_k4(b[:, 4:16])
    qh = b[:, 16:48]  # [nb, 32]
    qs = b[:, 48:176].reshape(-1, 4, 32)
    lo = np.stack([qs & 0x0F, qs >> 4], axis=2).reshape(-1, 8, 32).astype(np.int32)
    hbit = (qh[:, None, :].astype(np.int32) >> np.arange(8)[None, :, None]) & 1
    q = (lo | (hbit << 4)).astype(_f32)
    d1 = d[:, None] * sc.astype(_f32)
    m1 = dmin[:, None] * mn.astype(_f32)
    return (d1[:, :, None] * q - m1[:, :, None]).reshape(-1)


# ----------------------------------------------------------------------------------------
# Q6_K: [ql:128][qh:64][scales:int8 x16][d:f16] per 256 elements.
# Half n (128 elems) uses ql[64n:64n+64], qh[32n:32n+32], scales[8n:8n+8].
# For l<32: elem +l: ql[l]&15 | (qh[l]&3)<<4; +32: ql[l+32]&15 | ((qh[l]>>2)&3)<<4;
#           +64: ql[l]>>4 | ((qh[l]>>4)&3)<<4; +96: ql[l+32]>>4 | ((qh[l]>>6)&3)<<4.
# Stored q is offset by 32; w = d * scale[sub] * (q - 32), sub = element // 16.
# ----------------------------------------------------------------------------------------

def quantize_q6_k(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=_f32).reshape(-1, QK_K)
    nb = x.shape[0]
    xs = x.reshape(nb, 16, 16)
    idx = np.abs(xs).argmax(axis=2)
    vmax = np.take_along_axis(xs, idx[:, :, None], axis=2)[:, :, 0]
    scale = vmax / _f32(-32.0)
    d = (np.abs(scale).max(axis=1) / _f32(127.0)).astype(_f16)
    df = d.astype(_f32)
    sc = np.where(df[:, None] > 0, np.rint(scale / np.where(df > 0, df, _f32(1))[:, None]), 0)
    sc = np.clip(sc, -128, 127).astype(np.int32)
    eff = df[:, None] * sc.astype(_f32)
    safe = np.where(eff != 0, eff, _f32(1.0))
    q = np.rint(xs / safe[:, :, None])
    q = np.where(eff[:, :, None] != 0, q, 0)
    q = (np.clip(q, -32, 31).astype(np.int32) + 32).reshape(nb, 2, 4, 32)  # [nb, half, quarter, l]
    ql = np.empty((nb, 2, 64), np.int32)
    ql[:, :, 0:32] = (q[:, :, 0, :] & 15) | ((q[:, :, 2, :] & 15) << 4)
    ql[:, :, 32:64] = (q[:, :, 1, :] & 15) | ((q[:, :, 3, :] & 15) << 4)
    qh = ((q[:, :, 0, :] >> 4) | ((q[:, :, 1, :] >> 4) << 2) | ((q[:, :, 2, :] >> 4) << 4)
          | ((q[:, :, 3, :] >> 4) << 6))
    out = np.empty((nb, 210), np.uint8)
    out[:, 0:128] = ql.reshape(nb, 128).astype(np.uint8)
    out[:, 128:192] = qh.reshape(nb, 64).astype(np.uint8)
    out[:, 192:208] = sc.astype(np.int8).view(np.uint8)
    out[:, 208:210] = d.view(np.uint8).reshape(-1, 2)
    return out.reshape(-1)


def dequantize_q6_k(raw: np.ndarray) -> np.ndarray:
    b = _as_blocks(raw, 210)
    nb = b.shape[0]
    ql = b[:, 0:128].reshape(nb, 2, 64).astype(np.int32)
    qh = b[:, 128:192].reshape(nb, 2, 32).astype(np.int32)
    sc = b[:, 192:208].view(np.int8).astype(_f32).reshape(nb, 16)
    d = _f16_at(b, 208)
    q = np.empty((nb, 2, 4, 32), np.int32)
    q[:, :, 0] = (ql[:, :, 0:32] & 15) | ((qh & 3) << 4)
    q[:, :, 1] = (ql[:, :, 32:64] & 15) | (((qh >> 2) & 3) << 4)
    q[:, :, 2] = (ql[:, :, 0:32] >> 4) | (((qh >> 4) & 3) << 4)
    q[:, :, 3] = (ql[:, :, 32:64] >> 4) | (((qh >> 6) & 3) << 4)
    q = (q - 32).astype(_f32).reshape(nb, 16, 16)
    return (d[:, None, None] * sc[:, :, None] * q).reshape(-1)


def dequantize_q2_k(raw: np.ndarray) -> np.ndarray:
    b = _as_blocks(raw, 84)
    nb = b.shape[0]
    scales = b[:, 0:16].astype(np.int32)
    qs = b[:, 16:80].reshape(nb, 2, 32).astype(np.int32)
    d = _f16_at(b, 80)
    dmin = _f16_at(b, 82)
    out = np.empty((nb, 2, 4, 2, 16), _f32)
    for half in range(2):
        for j in range(4):
            sh = 2 * j
            for k in range(2):
                s = scales[:, half * 8 + j * 2 + k]
                dl = d * (s & 0xF).astype(_f32)
                ml = dmin * (s >> 4).astype(_f32)
                qq = ((qs[:, half, k * 16:(k + 1) * 16] >> sh) & 3).astype(_f32)
                out[:, half, j, k] = dl[:, None] * qq - ml[:, None]
    return out.reshape(-1)


# ----------------------------------------------------------------------------------------
# plain float formats
# ----------------------------------------------------------------------------------------

def bf16_to_f32(raw: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(raw).view(np.uint16).astype(np.uint32) << 16
    return u.view(_f32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=_f32).view(np.uint32)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return rounded.astype(np.uint16)


# ---- G4: group-wise asymmetric 4-bit (AWQ / GPTQ), groups of 128 --------------------------------
# 144 B per 256 weights: (s0, m0, s1, m1) as f32 then 128 B of codes laid out like Q4_K's qs
# (chunk c of 64 weights: byte b holds weight 64c+b in its low nibble and 64c+32+b in its high one).
# w = s_g * q - m_g with m_g = s_g * z_g, i.e. (q - z_g) * s_g of the AWQ/GPTQ checkpoints.
G4_GROUP = 128


def _g4_nibbles(codes: np.ndarray) -> np.ndarray:
    """codes [nb, 256] (0..15) -> [nb, 128] bytes in the Q4_K order."""
    c = codes.reshape(-1, 4, 2, 32).astype(np.uint8)
    return (c[:, :, 0, :] | (c[:, :, 1, :] << 4)).reshape(-1, 128)


def _g4_codes(qs: np.ndarray) -> np.ndarray:
    q = qs.reshape(-1, 4, 1, 32)
    return np.concatenate([q & 15, q >> 4], axis=2).reshape(-1, 256)


def g4_from_codes(codes: np.ndarray, scales: np.ndarray, zeros: np.ndarray, group: int) -> np.ndarray:
    """Rows of G4 blocks from per-weight codes [out, in] (0..15), scales / zero points [out, in/group].

    ``group`` must be a multiple of 128 (each 128-group of a block takes its group's pair)."""
    out_, in_ = codes.shape
    if group % G4_GROUP or in_ % QK_K:
        raise ValueError(f"G4 needs groups of a multiple of {G4_GROUP} and rows of a multiple of {QK_K}")
    rep = group // G4_GROUP
    s = np.repeat(np.asarray(scales, _f32), rep, axis=1).reshape(-1, 2)         # [out*in/256, 2]
    m = (np.repeat(np.asarray(zeros, _f32), rep, axis=1).reshape(-1, 2) * s).astype(_f32)
    hdr = np.stack([s[:, 0], m[:, 0], s[:, 1], m[:, 1]], axis=1).astype(_f32).view(np.uint8)
    qs = _g4_nibbles(np.asarray(codes).reshape(-1, QK_K))
    return np.concatenate([hdr, qs], axis=1).reshape(out_, -1)


def quantize_g4(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest asymmetric 4-bit per 128-group (scale (max - min) / 15, integer zero point)."""
    g = np.ascontiguousarray(x, _f32).reshape(-1, G4_GROUP)
    lo = np.minimum(g.min(axis=1), 0).astype(_f32)
    hi = np.maximum(g.max(axis=1), 0).astype(_f32)
    s = ((hi - lo) / _f32(15)).astype(_f32)
    s = np.where(s > 0, s, _f32(1)).astype(_f32)
    z = np.clip(np.rint(-lo / s), 0, 15).astype(_f32)
    q = np.clip(np.rint(g / s[:, None]) + z[:, None], 0, 15).astype(np.uint8)
    rows = g.shape[0] // 2
    return g4_from_codes(q.reshape(rows, QK_K), s.reshape(rows, 2), z.reshape(rows, 2), G4_GROUP).reshape(-1)


def dequantize_g4(raw: np.ndarray) -> np.ndarray:
    b = _as_blocks(raw, 144)
    hdr = np.ascontiguousarray(b[:, :16]).view(_f32)                               # [nb, 4]
    q = _g4_codes(b[:, 16:]).astype(_f32).reshape(-1, 2, G4_GROUP)
    s = hdr[:, [0, 2]][:, :, None]
    m = hdr[:, [1, 3]][:, :, None]
    return (s * q - m).astype(_f32).reshape(-1)


_DEQUANT = {
    GGMLType.Q8_0: dequantize_q8_0,
    GGMLType.Q4_0: dequantize_q4_0,
    GGMLType.Q4_1: dequantize_q4_1,
    GGMLType.Q5_0: dequantize_q5_0,
    GGMLType.Q5_1: dequantize_q5_1,
    GGMLType.Q2_K: dequantize_q2_k,
    GGMLType.Q4_K: dequantize_q4_k,
    GGMLType.Q5_K: dequantize_q5_k,
    GGMLType.Q6_K: dequantize_q6_k,
    GGMLType.G4: dequantize_g4,
}

_QUANT = {
    GGMLType.Q8_0: quantize_q8_0,
    GGMLType.Q4_K: quantize_q4_k,
    GGMLType.Q6_K: quantize_q6_k,
    GGMLType.G4: quantize_g4,
}

SUPPORTED_DEQUANT = frozenset(_DEQUANT) | {GGMLType.F32, GGMLType.F16, GGMLType.BF16}
DEVICE_RESIDENT_QUANTS = frozenset({GGMLType.Q8_0, GGMLType.Q4_K, GGMLType.Q6_K, GGMLType.G4})


def dequantize(raw: np.ndarray, ggml_type: int, shape: tuple[int, ...] | None = None) -> np.ndarray:
    """Decode a GGML tensor payload to float32 (row-major, innermost dim last)."""
    t = GGMLType(ggml_type)
    if t == GGMLType.F32:
        out = np.ascontiguousarray(raw).view(_f32).copy()
    elif t == GGMLType.F16:
        out = np.ascontiguousarray(raw).view(_f16).astype(_f32)
    elif t == GGMLType.BF16:
        out = bf16_to_f32(raw)
    elif t in _DEQUANT:
        out = _DEQUANT[t](raw)
    else:
        raise NotImplementedError(f"dequantize: GGML type {t.name} is not supported")
    return out.reshape(shape) if shape is not None else out


def quantize(x: np.ndarray, ggml_type: int) -> np.ndarray:
    """Encode float weights (innermost dim a multiple of the block size) to GGML bytes."""
    t = GGMLType(ggml_type)
    x = np.ascontiguousarray(x, dtype=_f32)
    if t == GGMLType.F32:
        return x.reshape(-1).view(np.uint8).copy()
    if t == GGMLType.F16:
        return x.astype(_f16).reshape(-1).view(np.uint8).copy()
    if t == GGMLType.BF16:
        return f32_to_bf16(x).reshape(-1).view(np.uint8).copy()
    if t not in _QUANT:
        raise NotImplementedError(f"quantize: GGML type {t.name} is not supported")
    blk = BLOCK_INFO[t][0]
    if x.shape[-1] % blk:
        raise ValueError(f"{t.name}: row length {x.shape[-1]} is not a multiple of {blk}")
    return _QUANT[t](x)
