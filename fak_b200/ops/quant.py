"""Device-side GGML block formats: row-pitched weight buffers, (de)quantization, GPU synthesis."""
from __future__ import annotations

import torch

from ..gguf.constants import BLOCK_INFO, GGMLType
from ._ext import ext

QT_F32, QT_F16, QT_Q8_0, QT_Q4_K, QT_Q6_K, QT_BF16, QT_G4 = 0, 1, 8, 12, 14, 30, 64
DEVICE_QTYPES = (QT_Q8_0, QT_Q4_K, QT_Q6_K, QT_G4)


def row_bytes(qtype: int, cols: int) -> int:
    blk, nb = BLOCK_INFO[GGMLType(qtype)]
    if cols % blk:
        raise ValueError(f"{GGMLType(qtype).name}: {cols} columns is not a multiple of {blk}")
    return cols // blk * nb


def row_pitch(qtype: int, cols: int) -> int:
    """Row stride on the device (blocks stay unchanged): the packed row rounded up to 16 bytes and
    then to 16 mod 128, so a 16-row tile copied as one contiguous span lands in shared memory with
    consecutive rows on different banks."""
    p = (row_bytes(qtype, cols) + 15) // 16 * 16
    while p % 128 != 16:
        p += 16
    return p


def quantize_blocks(x: torch.Tensor, qtype: int) -> torch.Tensor:
    """fp32 CUDA tensor -> GGML block bytes (identical to fak_b200.gguf.quants on CPU)."""
    return ext().quantize_blocks(x.contiguous().float(), int(qtype))


def dequantize_rows(w: torch.Tensor, qtype: int, rows: int, cols: int, pitch: int,
                    dtype: torch.dtype = torch.float32) -> torch.Tensor:
    return ext().dequantize_rows(w, int(qtype), int(rows), int(cols), int(pitch), dtype)


def synth_quantized(shape: tuple[int, ...], ggml_type: int, seed: int, std: float, ones: bool = False,
                    device: str = "cuda") -> torch.Tensor:
    """Random N(0, std) values generated and block-quantized on the GPU; returns packed GGML bytes."""
    n = 1
    for s in shape:
        n *= int(s)
    if ones:
        x = torch.ones(n, device=device, dtype=torch.float32)
    else:
        g = torch.Generator(device=device)
        g.manual_seed(int(seed) & 0x7FFFFFFFFFFFFFFF)
        x = torch.randn(n, generator=g, device=device, dtype=torch.float32).mul_(std)
    t = int(ggml_type)
    if t == QT_F32:
        return x.view(torch.uint8)
    if t == QT_F16:
        return x.half().view(torch.uint8)
    if t == QT_BF16:
        return x.bfloat16().view(torch.uint8)
    return quantize_blocks(x, t)


# ---- tile-packed layout of the decode GEMV ----------------------------------------------------
# Rows in tiles of 16, each row's blocks in 256-weight units; one (tile, unit) is a contiguous
# "unit tile" whose fields are split into planes.  Plane row ("slot") s holds tile row
# (s >> 1) + 8 (s & 1) (except the Q6_K qh plane, kept in tile-row order); 16-byte chunks of the
# quant planes are XOR-swizzled.  The block bytes are unchanged, only placed differently.
TILE_UNIT_BYTES = {QT_Q4_K: 2304, QT_Q6_K: 3360, QT_Q8_0: 4352, QT_G4: 2304}
SLOT_ROWS = [(s >> 1) + 8 * (s & 1) for s in range(16)]


def _swizzle(plane: torch.Tensor, key) -> torch.Tensor:
    """plane [..., 16 slots, C chunks, 16]: chunk position p of slot s holds chunk p ^ key(s)."""
    C = plane.shape[-2]
    idx = torch.tensor([[p ^ key(s) for p in range(C)] for s in range(16)], device=plane.device)
    return plane[..., torch.arange(16, device=plane.device)[:, None], idx, :]


def tile_pack(buf: torch.Tensor, qtype: int, rows: int, cols: int, pitch: int) -> torch.Tensor:
    """Row-pitched GGML rows -> tile-packed bytes [ceil(rows/16), ceil(cols/256), unit bytes]."""
    qtype = int(qtype)
    if qtype not in TILE_UNIT_BYTES:
        raise ValueError(f"tile_pack: unsupported block type {qtype}")
    T, U = -(-rows // 16), -(-cols // 256)
    rb = row_bytes(qtype, cols)
    m = buf[: rows * pitch].view(rows, pitch)[:, :rb]
    if qtype == QT_Q8_0:
        nblk = cols // 32
        blocks = torch.zeros(T * 16, U * 8, 34, dtype=torch.uint8, device=buf.device)
        blocks[:rows, :nblk] = m.reshape(rows, nblk, 34)
        x = blocks.view(T, 16, U, 8, 34).permute(0, 2, 1, 3, 4)[:, :, SLOT_ROWS]  # [T,U,16,8,34]
        d = x[..., :2].reshape(T, U, 16 * 16)
        qs = _swizzle(x[..., 2:].reshape(T, U, 16, 16, 16), lambda s: s & 6).reshape(T, U, 4096)
        planes = [qs, d]
    else:
        ub = 144 if qtype in (QT_Q4_K, QT_G4) else 210
        full = torch.zeros(T * 16, U * ub, dtype=torch.uint8, device=buf.device)
        full[:rows] = m
        x = full.view(T, 16, U, ub).permute(0, 2, 1, 3)[:, :, SLOT_ROWS]  # [T,U,16,ub]
        if qtype in (QT_Q4_K, QT_G4):  # 16-byte header (K-quant scales, or G4's two (s, m) pairs)
            hdr = x[..., :16].reshape(T, U, 256)
            qs = _swizzle(x[..., 16:144].reshape(T, U, 16, 8, 16), lambda s: s & 6).reshape(T, U, 2048)
            planes = [hdr, qs]
        else:
            ql = _swizzle(x[..., :128].reshape(T, U, 16, 8, 16), lambda s: (s >> 1) & 7).reshape(T, U, 2048)
            # qh rows in tile-row order (plane row r = tile row r), chunks swizzled by (r >> 1) & 3
            qh_rows = x[..., 128:192][:, :, [SLOT_ROWS.index(r) for r in range(16)]]
            qh = _swizzle(qh_rows.reshape(T, U, 16, 4, 16), lambda r: (r >> 1) & 3).reshape(T, U, 1024)
            sc = x[..., 192:208].reshape(T, U, 256)
            d = x[..., 208:210].reshape(T, U, 32)
            planes = [ql, qh, sc, d]
    out = torch.cat(planes, dim=-1).contiguous()
    assert out.shape[-1] == TILE_UNIT_BYTES[qtype]
    return out
