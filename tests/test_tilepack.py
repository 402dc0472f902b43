"""Tile-packed decode-GEMV layout (CPU).

``kernel_view`` re-derives every weight of a tile-packed matrix with the same slot, swizzle,
nibble and scale-table arithmetic the tgemv kernel uses, so a wrong address in either the packer
or the kernel's index math shows up here as a mismatch against the plain GGML dequantizer.
"""
import numpy as np
import pytest
import torch

from fak_b200.gguf.quants import dequantize, quantize
from fak_b200.ops.quant import QT_Q4_K, QT_Q6_K, QT_Q8_0, row_bytes, row_pitch, tile_pack


def _u16(b):
    return b[..., 0].astype(np.uint16) | (b[..., 1].astype(np.uint16) << 8)


def _half(b):
    return _u16(b).view(np.float16).astype(np.float32)


def _u32(b4):
    b4 = b4.astype(np.uint32)
    return b4[0] | (b4[1] << 8) | (b4[2] << 16) | (b4[3] << 24)


def _byte(w, i):
    return (int(w) >> (8 * i)) & 0xFF


def kernel_view(tp: np.ndarray, qtype: int) -> np.ndarray:
    """tile-packed bytes [T, U, UT] -> dequantized [T*16, U*256] as the kernel reads them."""
    T, U, _ = tp.shape
    out = np.zeros((T * 16, U * 256), np.float32)
    for ti in range(T):
        for u in range(U):
            wt = tp[ti, u]
            for g in range(8):
                for row_half, s in ((0, 2 * g), (1, 2 * g + 1)):
                    row = ti * 16 + g + 8 * row_half
                    for t in range(4):
                        if qtype == QT_Q4_K:
                            hdr = wt[16 * s:16 * s + 16]
                            d, dm = _half(hdr[0:2]), _half(hdr[2:4])
                            y, z, w = _u32(hdr[4:8]), _u32(hdr[8:12]), _u32(hdr[12:16])
                            for c in range(4):
                                q = 2 * c + (t >> 1)
                                off = 256 + 128 * s + 16 * (q ^ (s & 6)) + 8 * (t & 1)
                                qb = wt[off:off + 8]
                                for hi in range(2):
                                    j = 2 * c + hi
                                    jh, i = j >> 2, j & 3
                                    scw = ((w & 0x0F0F0F0F) | ((y >> 2) & 0x30303030)) if jh else (y & 0x3F3F3F3F)
                                    mw = (((w >> 4) & 0x0F0F0F0F) | ((z >> 2) & 0x30303030)) if jh else (z & 0x3F3F3F3F)
                                    a = d * _byte(scw, i) * (0.0625 if j & 1 else 1.0)
                                    mm = dm * _byte(mw, i)
                                    nib = (qb & 0xF0) if hi else (qb & 0x0F)
                                    k = u * 256 + 32 * j + 8 * t
                                    out[row, k:k + 8] = a * nib.astype(np.float32) - mm
                        elif qtype == QT_Q6_K:
                            d = _half(wt[3328 + 2 * s:3330 + 2 * s])
                            sc = wt[3072 + 16 * s:3088 + 16 * s].view(np.int8)
                            f8, f4 = s >> 1 & 7, s >> 1 & 3
                            for n in range(2):
                                for h in range(2):
                                    c1, c2, ch = 4 * n + h, 4 * n + 2 + h, 2 * n + h
                                    la0 = wt[128 * s + 16 * (c1 ^ f8) + 4 * t:][:4]
                                    la1 = wt[128 * s + 16 * (c2 ^ f8) + 4 * t:][:4]
                                    r = g + 8 * row_half  # qh plane: tile-row order
                                    ha = wt[2048 + 64 * r + 16 * (ch ^ ((r >> 1) & 3)) + 4 * t:][:4]
                                    for kk in range(4):
                                        la = la1 if kk & 1 else la0
                                        q = ((la >> (4 * (kk >> 1))) & 0xF) | (((ha >> (2 * kk)) & 3) << 4)
                                        e0 = 128 * n + 32 * kk + 16 * h
                                        out[row, u * 256 + e0 + 4 * t:u * 256 + e0 + 4 * t + 4] = \
                                            d * float(sc[e0 >> 4]) * (q.astype(np.float32) - 32)
                        else:
                            for b in range(8):
                                q = 2 * b + (t >> 1)
                                off = 256 * s + 16 * (q ^ (s & 6)) + 8 * (t & 1)
                                qs = wt[off:off + 8].view(np.int8).astype(np.float32)
                                dd = _half(wt[4096 + 16 * s + 2 * b:4096 + 16 * s + 2 * b + 2])
                                k = u * 256 + 32 * b + 8 * t
                                out[row, k:k + 8] = dd * qs
    return out


@pytest.mark.parametrize("qtype,rows,cols", [(QT_Q4_K, 37, 512), (QT_Q6_K, 21, 768), (QT_Q8_0, 19, 576)])
def test_kernel_view_matches_dequantizer(qtype, rows, cols):
    x = np.random.default_rng(qtype).standard_normal((rows, cols)).astype(np.float32)
    q = quantize(x, qtype)
    rb, p = row_bytes(qtype, cols), row_pitch(qtype, cols)
    buf = torch.zeros(rows * p + p + 256, dtype=torch.uint8)
    buf[:rows * p].view(rows, p)[:, :rb] = torch.from_numpy(np.ascontiguousarray(q).reshape(rows, rb))
    tp = tile_pack(buf, qtype, rows, cols, p).numpy()
    got = kernel_view(tp, qtype)[:rows, :cols]
    want = dequantize(q, qtype, rows * cols).reshape(rows, cols)
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-6)
    # padding rows / columns dequantize to zero
    full = kernel_view(tp, qtype)
    assert not full[rows:].any() and not full[:, cols:].any()
