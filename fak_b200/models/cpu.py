"""Load a GGUF checkpoint into the C++ CPU runtime (``fak_b200._cpu.CpuModel``).

Weights are handed over in their GGML block bytes (Q8_0 / Q4_K / Q6_K / f16 / f32); GGML
"llama" Q/K rows are restored to HF rotary order on the way, exactly as for the GPU loader.
"""
from __future__ import annotations

import importlib

import numpy as np

from ..gguf import GGMLType
from ..gguf.quants import dequantize
from .loader import iter_raw_tensors, open_model

_NATIVE = {GGMLType.F32: 0, GGMLType.F16: 1, GGMLType.Q8_0: 8, GGMLType.Q4_K: 12, GGMLType.Q6_K: 14}


def cpu_ext():
    try:
        return importlib.import_module("fak_b200._cpu")
    except ImportError as e:
        raise ImportError("fak_b200._cpu is not built: run `python setup.py build_ext --inplace`") from e


def load_cpu_model(path: str, act_quant: bool = True):
    g, cfg = open_model(path)
    if cfg.is_moe:
        raise NotImplementedError("the CPU runtime covers the dense decoder families")
    m = cpu_ext().CpuModel({"n_layers": cfg.n_layers, "d_model": cfg.d_model, "n_heads": cfg.n_heads,
                            "n_kv_heads": cfg.n_kv_heads, "head_dim": cfg.head_dim, "ffn_dim": cfg.ffn_dim,
                            "vocab_size": cfg.vocab_size, "rms_eps": cfg.rms_eps, "rope_theta": cfg.rope_theta},
                           act_quant)
    mats = {"attn_q.weight": "q", "attn_k.weight": "k", "attn_v.weight": "v", "attn_output.weight": "o",
            "ffn_gate.weight": "gate", "ffn_up.weight": "up", "ffn_down.weight": "down"}
    vecs = {"attn_norm.weight": "attn_norm", "ffn_norm.weight": "ffn_norm", "attn_q.bias": "q_bias",
            "attn_k.bias": "k_bias", "attn_v.bias": "v_bias", "attn_q_norm.weight": "q_norm",
            "attn_k_norm.weight": "k_norm"}

    def put_matrix(name, layer, shape, t, raw):
        qt = _NATIVE.get(GGMLType(t))
        if qt is None:  # other block types: convert to f32 rows
            raw = dequantize(raw.reshape(-1), t).astype(np.float32).view(np.uint8).reshape(shape[0], -1)
            qt = 0
        m.set_matrix(name, layer, qt, shape[0], shape[1], np.ascontiguousarray(raw).tobytes())

    for name, shape, t, raw in iter_raw_tensors(g, cfg):
        if name == "token_embd.weight":
            put_matrix("embed", -1, shape, t, raw)
            if cfg.tie_embeddings:
                put_matrix("lm_head", -1, shape, t, raw)
        elif name == "output.weight":
            put_matrix("lm_head", -1, shape, t, raw)
        elif name == "output_norm.weight":
            m.set_vector("final_norm", -1, dequantize(raw.reshape(-1), t).astype(np.float32).tolist())
        elif name.startswith("blk."):
            _, li, rest = name.split(".", 2)
            if rest in mats:
                put_matrix(mats[rest], int(li), shape, t, raw)
            elif rest in vecs:
                m.set_vector(vecs[rest], int(li), dequantize(raw.reshape(-1), t).astype(np.float32).tolist())
    g.close()
    return m, cfg
