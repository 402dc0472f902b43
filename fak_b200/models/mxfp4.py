"""MXFP4 (OCP microscaling FP4) weights, the format gpt-oss ships its expert matrices in.

A block of 32 consecutive input-axis values shares one E8M0 scale byte (value 2^(s - 127)); each
value is an FP4 E2M1 code (sign, 2 exponent bits, 1 mantissa bit: magnitudes 0, 0.5, 1, 1.5, 2,
3, 4, 6), two codes per byte, the lower nibble first.  Checkpoints store ``<name>_blocks`` uint8
[..., rows, K / 32, 16] and ``<name>_scales`` uint8 [..., rows, K / 32], rows being the matrix's
output features.

The device has no FP4 block type, so these layers are dequantized on load and take the
quant-on-load path like every other float checkpoint.

Reference: the MXFP4 expert tensors of gpt-oss checkpoints (internal/model/tensor_resolver.go:441-455).
"""
from __future__ import annotations

import numpy as np

# E2M1 code -> value (bit 3: sign)
FP4_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                       -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=np.float32)


def dequantize(blocks: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """blocks uint8 [..., G, 16], scales uint8 [..., G] -> float32 [..., G * 32]."""
    blocks = np.asarray(blocks, dtype=np.uint8)
    scales = np.asarray(scales, dtype=np.uint8)
    if blocks.shape[-1] != 16 or blocks.shape[:-1] != scales.shape:
        raise ValueError(f"MXFP4 blocks {blocks.shape} do not match scales {scales.shape}")
    vals = np.empty(blocks.shape[:-1] + (32,), dtype=np.float32)
    vals[..., 0::2] = FP4_VALUES[blocks & 0x0F]
    vals[..., 1::2] = FP4_VALUES[blocks >> 4]
    vals = np.ldexp(vals, scales.astype(np.int32)[..., None] - 127)
    return vals.reshape(blocks.shape[:-2] + (blocks.shape[-2] * 32,))


def quantize(w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Round-to-nearest MXFP4 of ``w`` [..., K] (K a multiple of 32): (blocks, scales).  The block
    scale is the power of two that brings the block's largest magnitude to at most 6."""
    w = np.asarray(w, dtype=np.float32)
    if w.shape[-1] % 32:
        raise ValueError("MXFP4 needs the input axis to be a multiple of 32")
    g = w.reshape(w.shape[:-1] + (w.shape[-1] // 32, 32))
    amax = np.abs(g).max(axis=-1)
    e = np.where(amax > 0, np.ceil(np.log2(np.maximum(amax, 1e-30) / 6.0)), -127).astype(np.int32)
    e = np.clip(e, -127, 127)
    x = g / np.ldexp(np.float32(1.0), e)[..., None]
    mags = FP4_VALUES[:8]
    code = np.abs(np.abs(x)[..., None] - mags).argmin(axis=-1).astype(np.uint8)
    code |= np.where(x < 0, 8, 0).astype(np.uint8)
    blocks = (code[..., 0::2] | (code[..., 1::2] << 4)).astype(np.uint8)
    return blocks, (e + 127).astype(np.uint8)
