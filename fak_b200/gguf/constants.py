"""GGUF container constants: metadata value types and GGML tensor block types.

The numeric codes are fixed by the GGUF file format (the format is shared by
every GGUF producer and consumer; the reference reads the same codes in
internal/ggufload/gguf.go).  Block sizes and byte sizes follow the on-disk
layouts that Q4_K/Q6_K/Q8_0 checkpoints use, which this framework keeps
unchanged on the GPU.
"""
from __future__ import annotations

import enum

GGUF_MAGIC = 0x46554747  # b"GGUF" little-endian
GGUF_VERSION = 3
GGUF_DEFAULT_ALIGNMENT = 32


class ValueType(enum.IntEnum):
    UINT8 = 0
    INT8 = 1
    UINT16 = 2
    INT16 = 3
    UINT32 = 4
    INT32 = 5
    FLOAT32 = 6
    BOOL = 7
    STRING = 8
    ARRAY = 9
    UINT64 = 10
    INT64 = 11
    FLOAT64 = 12


class GGMLType(enum.IntEnum):
    F32 = 0
    F16 = 1
    Q4_0 = 2
    Q4_1 = 3
    Q5_0 = 6
    Q5_1 = 7
    Q8_0 = 8
    Q8_1 = 9
    Q2_K = 10
    Q3_K = 11
    Q4_K = 12
    Q5_K = 13
    Q6_K = 14
    Q8_K = 15
    IQ4_NL = 20
    IQ4_XS = 23
    I8 = 24
    I16 = 25
    I32 = 26
    I64 = 27
    F64 = 28
    BF16 = 30
    # framework-internal (not a GGML type): group-wise asymmetric 4-bit, groups of 128 along the
    # row -- the AWQ / GPTQ weight format.  Block of 256 weights, 144 bytes:
    # [s0 f32][m0 f32][s1 f32][m1 f32][128 B of codes in the Q4_K nibble order], w = s_g * q - m_g
    G4 = 64


QK_K = 256

# (elements per block, bytes per block)
BLOCK_INFO: dict[GGMLType, tuple[int, int]] = {
    GGMLType.F32: (1, 4),
    GGMLType.F16: (1, 2),
    GGMLType.BF16: (1, 2),
    GGMLType.F64: (1, 8),
    GGMLType.I8: (1, 1),
    GGMLType.I16: (1, 2),
    GGMLType.I32: (1, 4),
    GGMLType.I64: (1, 8),
    GGMLType.Q4_0: (32, 18),
    GGMLType.Q4_1: (32, 20),
    GGMLType.Q5_0: (32, 22),
    GGMLType.Q5_1: (32, 24),
    GGMLType.Q8_0: (32, 34),
    GGMLType.Q8_1: (32, 36),
    GGMLType.Q2_K: (QK_K, 84),
    GGMLType.Q3_K: (QK_K, 110),
    GGMLType.Q4_K: (QK_K, 144),
    GGMLType.Q5_K: (QK_K, 176),
    GGMLType.Q6_K: (QK_K, 210),
    GGMLType.Q8_K: (QK_K, 292),
    GGMLType.IQ4_NL: (32, 18),
    GGMLType.IQ4_XS: (QK_K, 136),
    GGMLType.G4: (QK_K, 144),
}

# llama.cpp "file_type" codes that appear in general.file_type
FILE_TYPE_ALL_F32 = 0
FILE_TYPE_MOSTLY_F16 = 1
FILE_TYPE_MOSTLY_Q8_0 = 7
FILE_TYPE_MOSTLY_Q4_K_M = 15
FILE_TYPE_MOSTLY_Q6_K = 18
FILE_TYPE_MOSTLY_BF16 = 32


def tensor_nbytes(ggml_type: int, n_elements: int) -> int:
    blk, nb = BLOCK_INFO[GGMLType(ggml_type)]
    if n_elements % blk:
        raise ValueError(f"{GGMLType(ggml_type).name}: {n_elements} elements is not a multiple of block {blk}")
    return n_elements // blk * nb


def row_nbytes(ggml_type: int, row_elements: int) -> int:
    return tensor_nbytes(ggml_type, row_elements)
