"""GGUF -> canonical tensors.

Two consumers:

* ``load_reference_tensors`` dequantizes everything to fp32 for the oracle
  (reference: ggufload.LoadModel, internal/ggufload/gguf_weightsource.go:16).
* ``iter_raw_tensors`` yields the stored GGML bytes unchanged, which the GPU
  weight uploader (models/weights.py) places on the device as-is
  (reference: the resident Q4_K/Q6_K path, internal/ggufload/quant_q4k_loader.go).

GGML's "llama" architecture stores Q/K rows in interleaved-rotary order; both
paths restore HF order by permuting whole rows, which is exact for quantized
rows (reference: unpermuteRotaryTensor, internal/ggufload/gguf_tensor_canonical.go:232).
"""
from __future__ import annotations

import os
from typing import Iterator

import numpy as np
import torch

from ..config import ModelConfig, config_from_gguf_metadata
from ..gguf import GGMLType, GGUFFile, open_gguf
from ..gguf.quants import dequantize


def llama_rope_unpermute_rows(rows: np.ndarray, n_heads: int, head_dim: int) -> np.ndarray:
    half = head_dim // 2
    r = rows.reshape(n_heads, half, 2, -1)
    return np.ascontiguousarray(r.transpose(0, 2, 1, 3)).reshape(rows.shape)


def _needs_unpermute(cfg: ModelConfig, name: str) -> int:
    if cfg.arch != "llama":
        return 0
    if name.endswith("attn_q.weight"):
        return cfg.n_heads
    if name.endswith("attn_k.weight"):
        return cfg.n_kv_heads
    return 0


def open_model(path_or_file: str | os.PathLike | GGUFFile) -> tuple[GGUFFile, ModelConfig]:
    g = path_or_file if isinstance(path_or_file, GGUFFile) else open_gguf(path_or_file)
    cfg = config_from_gguf_metadata(g.metadata, {k: v.shape for k, v in g.tensors.items()})
    return g, cfg


def iter_raw_tensors(g: GGUFFile, cfg: ModelConfig) -> Iterator[tuple[str, tuple[int, ...], GGMLType, np.ndarray]]:
    """(name, shape, ggml type, [rows, row_bytes] uint8) in HF row order."""
    for ti in g:
        raw = g.raw_rows(ti.name) if len(ti.shape) >= 2 else g.raw(ti.name).reshape(1, -1)
        heads = _needs_unpermute(cfg, ti.name)
        if heads:
            raw = llama_rope_unpermute_rows(raw, heads, cfg.head_dim)
        yield ti.name, ti.shape, ti.ggml_type, raw


def load_reference_tensors(path_or_file) -> tuple[ModelConfig, dict[str, torch.Tensor]]:
    g, cfg = open_model(path_or_file)
    out: dict[str, torch.Tensor] = {}
    for name, shape, t, raw in iter_raw_tensors(g, cfg):
        out[name] = torch.from_numpy(dequantize(raw, t, shape).astype(np.float32))
    return cfg, out
