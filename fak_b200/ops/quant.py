"""Device-side GGML block formats: row-pitched weight buffers, (de)quantization, GPU synthesis."""
from __future__ import annotations

import torch

from ..gguf.constants import BLOCK_INFO, GGMLType
from ._ext import ext

QT_F32, QT_F16, QT_Q8_0, QT_Q4_K, QT_Q6_K, QT_BF16 = 0, 1, 8, 12, 14, 30
DEVICE_QTYPES = (QT_Q8_0, QT_Q4_K, QT_Q6_K)


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
