"""EXL2 (ExLlamaV2) mixed-precision weights: each linear layer's input axis is split into groups
quantized at their own bit width (2-8 bits), so salient channels get more bits at a target average.

Storage per linear ``<name>`` (safetensors):

* ``q_groups``    int16 [2G]: (bits, size) per input-axis group, groups contiguous in storage order;
* ``q_weight``    int32 [out, words]: per output row, the codes of all storage columns packed
  least-significant-bit first into a continuous bit stream (a code may straddle two words);
* ``q_scale``     f16 [out, G] and ``q_scale_max`` f16 [G]: scale[o, g] = q_scale[o, g] * q_scale_max[g];
* ``q_invperm``   int32 [in]: logical input channel of each storage column (act-order), optional.

w[o, invperm[i]] = scale[o, g(i)] * (code[o, i] - 2^(bits_g - 1)).

The device has no mixed-width block type, so EXL2 layers are dequantized on load (vectorised over
whole groups) and take the quant-on-load path to Q8_0.

Reference: internal/model/exl2.go (storage contract, LSB-first variable-width packing, two-level
scale, inverse permutation).
"""
from __future__ import annotations

import numpy as np


def _bit_layout(groups: list[tuple[int, int]]) -> tuple[np.ndarray, np.ndarray, np.ndarray, int]:
    """Per storage column: bit width, bit position in the row stream, group index; words per row."""
    bits = np.concatenate([np.full(size, b, np.int64) for b, size in groups])
    gidx = np.concatenate([np.full(size, g, np.int64) for g, (_, size) in enumerate(groups)])
    pos = np.concatenate([[0], np.cumsum(bits)[:-1]]).astype(np.int64)
    words = int((int(bits.sum()) + 31) // 32)
    return bits, pos, gidx, words


def pack(codes: np.ndarray, groups: list[tuple[int, int]]) -> np.ndarray:
    """codes [out, in] (storage column order) -> q_weight int32 [out, words]."""
    out_, in_ = codes.shape
    bits, pos, _, words = _bit_layout(groups)
    if int(bits.size) != in_:
        raise ValueError("group sizes do not add up to the input width")
    acc = np.zeros((out_, words + 1), dtype=np.uint64)
    c = codes.astype(np.uint64)
    w, off = pos >> 5, (pos & 31).astype(np.uint64)
    lo = (c << off[None, :]) & np.uint64(0xFFFFFFFF)
    hi = c >> (np.uint64(32) - off[None, :])
    for i in range(in_):   # scatter-or; columns sharing a word are distinct bit ranges
        acc[:, w[i]] |= lo[:, i]
        if int(off[i]) + int(bits[i]) > 32:
            acc[:, w[i] + 1] |= hi[:, i]
    return acc[:, :words].astype(np.uint32).view(np.int32)


def unpack(q_weight: np.ndarray, groups: list[tuple[int, int]]) -> np.ndarray:
    """q_weight [out, words] -> codes [out, in] (storage column order)."""
    bits, pos, _, words = _bit_layout(groups)
    wds = np.ascontiguousarray(q_weight).view(np.uint32).astype(np.uint64)
    wds = np.concatenate([wds, np.zeros((wds.shape[0], 1), np.uint64)], axis=1)
    w, off = pos >> 5, (pos & 31).astype(np.uint64)
    x = wds[:, w] | (wds[:, w + 1] << np.uint64(32))
    mask = (np.uint64(1) << bits.astype(np.uint64)) - np.uint64(1)
    return ((x >> off[None, :]) & mask[None, :]).astype(np.int64)


def dequantize(q_weight, q_groups, q_scale, q_scale_max, q_invperm=None) -> np.ndarray:
    """float32 [out, in] in logical input order."""
    g = np.asarray(q_groups).astype(np.int64).reshape(-1, 2)
    groups = [(int(b), int(s)) for b, s in g]
    codes = unpack(q_weight, groups)
    bits, _, gidx, _ = _bit_layout(groups)
    scale = np.asarray(q_scale, np.float32) * np.asarray(q_scale_max, np.float32)[None, :]
    w = (scale[:, gidx] * (codes - (np.int64(1) << (bits - 1))[None, :]).astype(np.float32)).astype(np.float32)
    if q_invperm is None:
        return w
    out = np.empty_like(w)
    out[:, np.asarray(q_invperm, np.int64)] = w
    return out


def quantize(w: np.ndarray, groups: list[tuple[int, int]], perm: np.ndarray | None = None):
    """Round-to-nearest EXL2 tensors of ``w`` [out, in]: storage column i holds logical channel
    perm[i] (identity when None).  Returns (q_weight, q_groups, q_scale, q_scale_max, q_invperm)."""
    out_, in_ = w.shape
    perm = np.arange(in_) if perm is None else np.asarray(perm, np.int64)
    ws = w[:, perm].astype(np.float32)
    bits, _, gidx, _ = _bit_layout(groups)
    G = len(groups)
    amax = np.stack([np.abs(ws[:, gidx == g]).max(axis=1) for g in range(G)], axis=1)     # [out, G]
    half = np.array([(1 << (b - 1)) - 1 if b > 1 else 1 for b, _ in groups], np.float32)
    s = np.maximum(amax / half[None, :], 1e-12).astype(np.float32)
    smax = s.max(axis=0).astype(np.float16).astype(np.float32)
    q_scale = (s / smax[None, :]).astype(np.float16)
    scale = q_scale.astype(np.float32) * smax[None, :]
    center = (np.int64(1) << (bits - 1))
    codes = np.clip(np.rint(ws / scale[:, gidx]) + center[None, :], 0, (np.int64(1) << bits) - 1).astype(np.int64)
    q_groups = np.array([x for b, size in groups for x in (b, size)], np.int16)
    # q_invperm[i]: the logical channel storage column i holds
    return pack(codes, groups), q_groups, q_scale, smax.astype(np.float16), perm.astype(np.int32)
