"""Hugging Face checkpoints: safetensors shards + config.json as a weight source.

``hf_source(dir)`` returns the same (config, getter, close) triple as the GGUF source, with tensors
renamed to the GGUF names the loaders use and float matrices handed over unquantized, so
``load_weights`` quantizes them to Q8_0 on load (the reference's quant-on-load path) and the fp32
reference model reads them as they are.  HF stores q/k rows in rotate_half order already (no
GGML "llama" permutation to undo).  Expert weights of Qwen3-MoE checkpoints (one tensor per
expert) are stacked into the [E, rows, cols] tensors of the GGUF layout.

The safetensors container is read directly (8-byte little-endian header length, JSON header of
{name: {dtype, shape, data_offsets}}, raw little-endian data) through a memory map.

Reference: safetensors loading and HF config parsing (internal/model/weights.go:333, Load;
internal/model/config.go:374-605), quant-on-load (internal/ggufload/gguf_weightsource.go:35-60).
"""
from __future__ import annotations

import glob
import json
import os
import re
import struct
from typing import Callable

import numpy as np
import torch

from ..config import ModelConfig
from ..gguf import GGMLType

_NP = {"F32": np.float32, "F16": np.float16, "BF16": np.uint16, "I32": np.int32, "I64": np.int64, "U8": np.uint8,
       "I8": np.int8, "I16": np.int16}
_GG = {"F32": GGMLType.F32, "F16": GGMLType.F16, "BF16": GGMLType.BF16}


def read_safetensors(path: str) -> dict[str, tuple[str, tuple[int, ...], np.ndarray]]:
    """name -> (dtype, shape, memory-mapped array of the raw elements)."""
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    base = 8 + n
    out = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        a, b = info["data_offsets"]
        dt = info["dtype"]
        if dt not in _NP:
            raise ValueError(f"{path}: unsupported safetensors dtype {dt} for {name}")
        arr = mm[base + a:base + b].view(_NP[dt]).reshape(info["shape"] or [1])
        out[name] = (dt, tuple(info["shape"]), arr)
    return out


def write_safetensors(path: str, tensors: dict[str, torch.Tensor], metadata: dict | None = None) -> None:
    """Write float32/float16/bfloat16 (and int32/int64/uint8/int8) tensors in the safetensors layout."""
    names = sorted(tensors)
    header, blobs, off = {}, [], 0
    for n in names:
        t = tensors[n].detach().cpu().contiguous()
        dt = {torch.float32: "F32", torch.float16: "F16", torch.bfloat16: "BF16", torch.int32: "I32",
              torch.int64: "I64", torch.uint8: "U8", torch.int8: "I8"}[t.dtype]
        raw = t.view(torch.uint16).numpy().tobytes() if t.dtype == torch.bfloat16 else t.numpy().tobytes()
        header[n] = {"dtype": dt, "shape": list(t.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    if metadata:
        header["__metadata__"] = {k: str(v) for k, v in metadata.items()}
    hb = json.dumps(header).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for b in blobs:
            f.write(b)


def config_from_hf(hf: dict) -> ModelConfig:
    arch_name = (hf.get("architectures") or [hf.get("model_type", "")])[0].lower()
    if isinstance(hf.get("text_config"), dict):   # multimodal wrapper: the text decoder's config
        hf = {**hf["text_config"], "architectures": hf.get("architectures")}
    mt = str(hf.get("model_type") or "")
    if "qwen3_5" in arch_name or mt.startswith("qwen3_5"):
        if "moe" in arch_name or "moe" in mt:
            raise ValueError("Qwen3.5-MoE is not supported (the dense Qwen3.5 hybrid is)")
        arch = "qwen35"
    elif "gemma2" in arch_name or hf.get("model_type") == "gemma2":
        arch = "gemma2"
    elif "gptoss" in arch_name or hf.get("model_type") == "gpt_oss":
        arch = "gptoss"
    elif "qwen3moe" in arch_name or hf.get("model_type") == "qwen3_moe":
        arch = "qwen3moe"
    elif "qwen3" in arch_name:
        arch = "qwen3"
    elif "qwen2" in arch_name:
        arch = "qwen2"
    elif "llama" in arch_name or "mistral" in arch_name or "phi3" in arch_name:
        arch = "llama"   # Phi-3: fused qkv / gate_up projections are split on load
    else:
        raise ValueError(f"unsupported HF architecture {arch_name!r}")
    d, H = int(hf["hidden_size"]), int(hf["num_attention_heads"])
    rp = hf.get("rope_parameters") or hf.get("rope_scaling") or {}   # v5 configs nest rope_theta here
    theta = float(hf.get("rope_theta") or rp.get("rope_theta") or 10000.0)
    cfg = ModelConfig(
        arch=arch, n_layers=int(hf["num_hidden_layers"]), d_model=d, n_heads=H,
        n_kv_heads=int(hf.get("num_key_value_heads", H)), head_dim=int(hf.get("head_dim") or d // H),
        ffn_dim=int(hf.get("intermediate_size", 0)), vocab_size=int(hf["vocab_size"]),
        rms_eps=float(hf.get("rms_norm_eps", 1e-6)), rope_theta=theta,
        tie_embeddings=bool(hf.get("tie_word_embeddings", False)),
        qkv_bias=arch == "qwen2" or (arch == "gptoss" and bool(hf.get("attention_bias", True))),
        qk_norm=arch in ("qwen3", "qwen3moe", "qwen35"),
        **(_gptoss_fields(hf) if arch == "gptoss" else {
            "n_experts": int(hf.get("num_experts", 0)) if arch == "qwen3moe" else 0,
            "n_experts_used": int(hf.get("num_experts_per_tok", 0)) if arch == "qwen3moe" else 0,
            "expert_ffn_dim": int(hf.get("moe_intermediate_size", 0)) if arch == "qwen3moe" else 0}),
        norm_topk_prob=bool(hf.get("norm_topk_prob", True)),
        max_context=int(hf.get("max_position_embeddings", 32768)),
        rope_scaling=_hf_rope_scaling(rp, hf),
        **(_gemma_fields(hf) if arch == "gemma2" else {}),
        **(_qwen35_fields(hf, rp) if arch == "qwen35" else {}),
        **_hf_sliding_window(hf, int(hf["num_hidden_layers"])),
        bos_token_id=int(hf.get("bos_token_id") or 1), eos_token_id=int(hf.get("eos_token_id") or 2),
        name=str(hf.get("_name_or_path", arch_name)),
    )
    cfg.validate()
    return cfg


def _gemma_fields(hf: dict) -> dict:
    act = str(hf.get("hidden_activation") or hf.get("hidden_act") or "gelu_pytorch_tanh")
    return {"act": "gelu_tanh" if "gelu" in act else "silu",
            "attn_softcap": float(hf.get("attn_logit_softcapping") or 0.0),
            "final_softcap": float(hf.get("final_logit_softcapping") or 0.0),
            "sandwich_norms": True, "embed_scale": float(hf["hidden_size"]) ** 0.5,
            "attn_scale": float(hf.get("query_pre_attn_scalar") or hf.get("head_dim") or 256) ** -0.5}


def _qwen35_fields(hf: dict, rp: dict) -> dict:
    """Qwen3.5 hybrid: "linear_attention" layers run Gated DeltaNet; full-attention layers have a
    sigmoid output gate and rotate partial_rotary_factor of each head."""
    types = hf.get("layer_types") or []
    hd = int(hf.get("head_dim") or hf["hidden_size"] // hf["num_attention_heads"])
    prf = float(rp.get("partial_rotary_factor") or hf.get("partial_rotary_factor") or 1.0)
    return {"linear_layers": tuple(i for i, t in enumerate(types) if t == "linear_attention"),
            "gdn_conv": int(hf.get("linear_conv_kernel_dim", 4)),
            "gdn_k_heads": int(hf["linear_num_key_heads"]), "gdn_v_heads": int(hf["linear_num_value_heads"]),
            "gdn_k_dim": int(hf["linear_key_head_dim"]), "gdn_v_dim": int(hf["linear_value_head_dim"]),
            "attn_out_gate": True, "rotary_dim": int(hd * prf)}


def _gptoss_fields(hf: dict) -> dict:
    """gpt-oss: every layer routed (num_local_experts, top num_experts_per_tok, width
    intermediate_size), attention sinks, biased projections, router and experts, clamped OAI gate."""
    bias = bool(hf.get("attention_bias", True))
    return {"n_experts": int(hf["num_local_experts"]), "n_experts_used": int(hf["num_experts_per_tok"]),
            "expert_ffn_dim": int(hf["intermediate_size"]), "attn_sinks": True, "attn_out_bias": bias,
            "router": "topk_softmax", "moe_bias": True, "swiglu_alpha": 1.702,
            "swiglu_limit": float(hf.get("swiglu_limit") or 7.0)}


def _hf_sliding_window(hf: dict, n_layers: int) -> dict:
    """Mistral: ``sliding_window`` on every layer; Qwen2: ``use_sliding_window`` from layer
    ``max_window_layers`` on; configs with ``layer_types``: the "sliding_attention" layers."""
    w = int(hf.get("sliding_window") or 0)
    if w <= 0:
        return {}
    types = hf.get("layer_types")
    if types:
        layers = tuple(i for i, t in enumerate(types) if t == "sliding_attention")
        return {"sliding_window": w, "swa_layers": layers} if layers else {}
    if "use_sliding_window" in hf:
        if not hf["use_sliding_window"]:
            return {}
        first = int(hf.get("max_window_layers", 0) or 0)
        return {"sliding_window": w, "swa_layers": tuple(range(first, n_layers))}
    return {"sliding_window": w}


def _hf_rope_scaling(rs: dict | None, hf: dict | None = None) -> dict | None:
    if not rs:
        return None
    kind = str(rs.get("rope_type") or rs.get("type") or "default").lower()
    if kind == "default":
        return None
    out = {k: v for k, v in rs.items() if k not in ("rope_type", "type", "rope_theta") and v is not None}
    out["type"] = kind
    if hf and "original_max_position_embeddings" not in out and hf.get("original_max_position_embeddings"):
        out["original_max_position_embeddings"] = int(hf["original_max_position_embeddings"])   # Phi-3
    return out


_LAYER = {
    "self_attn.q_proj.weight": "attn_q.weight", "self_attn.k_proj.weight": "attn_k.weight",
    "self_attn.v_proj.weight": "attn_v.weight", "self_attn.o_proj.weight": "attn_output.weight",
    "self_attn.q_proj.bias": "attn_q.bias", "self_attn.k_proj.bias": "attn_k.bias",
    "self_attn.v_proj.bias": "attn_v.bias", "self_attn.q_norm.weight": "attn_q_norm.weight",
    "self_attn.k_norm.weight": "attn_k_norm.weight", "input_layernorm.weight": "attn_norm.weight",
    "post_attention_layernorm.weight": "ffn_norm.weight", "mlp.gate_proj.weight": "ffn_gate.weight",
    "mlp.up_proj.weight": "ffn_up.weight", "mlp.down_proj.weight": "ffn_down.weight",
    "mlp.gate.weight": "ffn_gate_inp.weight",
    # gpt-oss
    "self_attn.sinks": "attn_sinks.weight", "self_attn.o_proj.bias": "attn_output.bias",
    "mlp.router.weight": "ffn_gate_inp.weight", "mlp.router.bias": "ffn_gate_inp.bias",
    # Qwen3.5 Gated DeltaNet layers
    "linear_attn.in_proj_qkv.weight": "ssm_in_qkv.weight", "linear_attn.in_proj_z.weight": "ssm_in_z.weight",
    "linear_attn.in_proj_b.weight": "ssm_in_b.weight", "linear_attn.in_proj_a.weight": "ssm_in_a.weight",
    "linear_attn.conv1d.weight": "ssm_conv1d.weight", "linear_attn.dt_bias": "ssm_dt.bias",
    "linear_attn.A_log": "ssm_a", "linear_attn.norm.weight": "ssm_norm.weight",
    "linear_attn.out_proj.weight": "ssm_out.weight",
}
# gpt-oss experts: all experts of a layer in one tensor; gate and up rows interleaved (gate even)
_FUSED_EXPERTS = re.compile(r"model\.layers\.(\d+)\.mlp\.experts\.(gate_up_proj|down_proj)(_blocks|_scales|_bias)?")
_EXPERT = re.compile(r"model\.layers\.(\d+)\.mlp\.experts\.(\d+)\.(gate|up|down)_proj\.weight")
_EXP_NAME = {"gate": "ffn_gate_exps.weight", "up": "ffn_up_exps.weight", "down": "ffn_down_exps.weight"}


_GEMMA_LAYER = {"post_attention_layernorm.weight": "post_attention_norm.weight",
                "pre_feedforward_layernorm.weight": "ffn_norm.weight",
                "post_feedforward_layernorm.weight": "post_ffw_norm.weight"}


def gguf_name(hf_name: str, arch: str = "") -> str | None:
    if hf_name == "model.embed_tokens.weight":
        return "token_embd.weight"
    if hf_name == "model.norm.weight":
        return "output_norm.weight"
    if hf_name == "lm_head.weight":
        return "output.weight"
    m = re.fullmatch(r"model\.layers\.(\d+)\.(.+)", hf_name)
    if m and arch == "gemma2" and m.group(2) in _GEMMA_LAYER:
        return f"blk.{m.group(1)}.{_GEMMA_LAYER[m.group(2)]}"
    if m and m.group(2) in _LAYER:
        return f"blk.{m.group(1)}.{_LAYER[m.group(2)]}"
    return None


def _to_f32(dt: str, a: np.ndarray) -> np.ndarray:
    if dt == "BF16":
        return (a.astype(np.uint32) << 16).view(np.float32)
    return a.astype(np.float32)


_QPARTS = (".qweight", ".qzeros", ".scales", ".g_idx")
_EXL2_PARTS = (".q_weight", ".q_groups", ".q_scale", ".q_scale_max", ".q_invperm")


def _quant_config(hf: dict) -> dict | None:
    q = hf.get("quantization_config")
    if not q:
        return None
    method = str(q.get("quant_method", "")).lower()
    if method in ("exl2", "mxfp4"):
        return None   # recognised by their tensors (q_groups, q_weight, ... / _blocks, _scales)
    if method not in ("awq", "gptq"):
        raise ValueError(f"unsupported quantization method {method!r} (AWQ, GPTQ, EXL2 and MXFP4 are)")
    return q


def _decode_quantized(qc: dict, parts: dict[str, np.ndarray]) -> tuple[tuple[int, int], int, np.ndarray]:
    """One qweight/qzeros/scales[/g_idx] triple -> ((out, in), ggml type, rows)."""
    from . import quantized_ckpt as qk
    bits, group = int(qc.get("bits", 4)), int(qc.get("group_size", 128))
    if qc["quant_method"].lower() == "awq":
        if bits != 4:
            raise ValueError("AWQ checkpoints are 4-bit")
        n_in = parts["qweight"].shape[0]
        group = n_in if group <= 0 else group
        codes, sc, z, _ = qk.unpack_awq(parts["qweight"], parts["qzeros"], _f32s(parts["scales"]), group)
        gidx = np.arange(n_in) // group
    else:
        n_in = parts["qweight"].shape[0] * 32 // bits
        group = n_in if group <= 0 else group
        v1 = str(qc.get("checkpoint_format", "gptq")).lower() != "gptq_v2"
        codes, sc, z, gidx = qk.unpack_gptq(parts["qweight"], parts["qzeros"], _f32s(parts["scales"]),
                                           parts.get("g_idx"), bits, group, v1)
    rows, t = qk.device_rows(codes, sc, z, gidx, group, bits)
    return codes.shape, t, rows


def _f32s(a: tuple[str, np.ndarray] | np.ndarray) -> np.ndarray:
    dt, arr = a
    return _to_f32(dt, np.asarray(arr))


def hf_source(model_dir: str) -> tuple[ModelConfig, Callable, Callable[[], None]]:
    with open(os.path.join(model_dir, "config.json")) as f:
        hfcfg = json.load(f)
    cfg = config_from_hf(hfcfg)
    qc = _quant_config(hfcfg)
    files = sorted(glob.glob(os.path.join(model_dir, "*.safetensors")))
    if not files:
        raise FileNotFoundError(f"no *.safetensors in {model_dir}")
    table: dict[str, tuple[str, tuple[int, ...], np.ndarray]] = {}
    experts: dict[str, dict[int, tuple[str, np.ndarray]]] = {}
    qparts: dict[str, dict[str, object]] = {}   # base name -> {qweight, qzeros, scales, g_idx}
    exl2_parts: dict[str, dict[str, tuple]] = {}   # base name -> {q_weight, q_groups, q_scale, ...}
    fused: dict[tuple[str, str], dict[str, tuple]] = {}   # (layer, gate_up_proj | down_proj) -> parts
    for p in files:
        for n, (dt, shape, arr) in read_safetensors(p).items():
            if qc is not None and n.endswith(_QPARTS):
                base, part = n.rsplit(".", 1)
                qparts.setdefault(base, {})[part] = (dt, arr) if part == "scales" else np.asarray(arr)
                continue
            if n.endswith(_EXL2_PARTS):
                base, part = n.rsplit(".", 1)
                exl2_parts.setdefault(base, {})[part] = (dt, np.asarray(arr))
                continue
            m = _EXPERT.fullmatch(n)
            if m:
                key = f"blk.{m.group(1)}.{_EXP_NAME[m.group(3)]}"
                experts.setdefault(key, {})[int(m.group(2))] = (dt, arr)
                continue
            m = _FUSED_EXPERTS.fullmatch(n)
            if m:
                fused.setdefault((m.group(1), m.group(2)), {})[m.group(3) or ""] = (dt, np.asarray(arr))
                continue
            m2 = re.fullmatch(r"model\.layers\.(\d+)\.(self_attn\.qkv_proj|mlp\.gate_up_proj)\.weight", n)
            if m2:   # fused projections: row ranges of one matrix
                i = m2.group(1)
                if m2.group(2) == "self_attn.qkv_proj":
                    q, kv = cfg.q_dim, cfg.kv_dim
                    parts = (("attn_q", 0, q), ("attn_k", q, q + kv), ("attn_v", q + kv, q + 2 * kv))
                else:
                    f = shape[0] // 2
                    parts = (("ffn_gate", 0, f), ("ffn_up", f, 2 * f))
                for nm, a, b in parts:
                    sub = arr[a:b]
                    table[f"blk.{i}.{nm}.weight"] = (dt, (b - a,) + tuple(shape[1:]), sub)
                continue
            g = gguf_name(n, cfg.arch)
            if g is not None:
                if g.endswith("norm.weight") and (cfg.arch == "gemma2" or (
                        cfg.arch == "qwen35" and not g.endswith("ssm_norm.weight"))):   # scaled by (1 + w)
                    arr = _to_f32(dt, np.asarray(arr)) + np.float32(1.0)
                    dt = "F32"
                if g.endswith("ssm_conv1d.weight"):   # [C, 1, K] -> [C, K]
                    shape = (shape[0], shape[-1])
                    arr = np.asarray(arr).reshape(shape)
                table[g] = (dt, shape, arr)
    # quantized layers: decoded on first use; experts (one triple per expert) stacked
    qlayers: dict[str, list[dict]] = {}
    for base, parts in qparts.items():
        if "qweight" not in parts:
            continue
        m = _EXPERT.fullmatch(base + ".weight")
        if m:
            key = f"blk.{m.group(1)}.{_EXP_NAME[m.group(3)]}"
            lst = qlayers.setdefault(key, [])
            lst.extend([None] * (int(m.group(2)) + 1 - len(lst)))
            lst[int(m.group(2))] = parts
            continue
        g = gguf_name(base + ".weight")
        if g is not None:
            qlayers[g] = [parts]
    for base, parts in exl2_parts.items():   # mixed-precision layers: float32 rows (quantized on load)
        g = gguf_name(base + ".weight")
        if g is None or "q_weight" not in parts:
            continue
        from . import exl2
        f = lambda k: _to_f32(*parts[k]) if parts[k][0] in ("F16", "BF16", "F32") else parts[k][1]
        w = exl2.dequantize(parts["q_weight"][1], parts["q_groups"][1], f("q_scale"), f("q_scale_max"),
                            parts["q_invperm"][1] if "q_invperm" in parts else None)
        table[g] = ("F32", tuple(w.shape), w)
    for (i, kind), parts in fused.items():
        table.update(_fused_experts(i, kind, parts))
    for key, per in experts.items():
        dts = {d for d, _ in per.values()}
        stacked = np.stack([per[e][1] for e in range(len(per))])
        table[key] = (dts.pop(), stacked.shape, stacked)
    if cfg.tie_embeddings or ("output.weight" not in table and "output.weight" not in qlayers):
        cfg = cfg.replace(tie_embeddings=True)

    def get(name: str):
        if name in qlayers:
            dec = [_decode_quantized(qc, parts) for parts in qlayers[name]]
            types = {t for _, t, _ in dec}
            if len(types) > 1:   # mixed layouts across experts: every one as float32
                dec = [(sh, int(GGMLType.F32), np.ascontiguousarray(
                    _dequant_rows(r, t, sh))) for sh, t, r in dec]
            (o, i), t, _ = dec[0]
            rows = np.concatenate([r for _, _, r in dec]) if len(dec) > 1 else dec[0][2]
            shape = (len(dec), o, i) if len(dec) > 1 else (o, i)
            return shape, int(dec[0][1]), torch.from_numpy(np.ascontiguousarray(rows).view(np.uint8))
        if name not in table:
            raise KeyError(f"{model_dir}: no tensor for {name}")
        dt, shape, arr = table[name]
        if dt not in _GG:
            raise ValueError(f"{name}: dtype {dt} is not a float type")
        a = np.ascontiguousarray(arr)
        rows = int(np.prod(shape[:-1])) if len(shape) > 1 else 1
        return tuple(shape), int(_GG[dt]), torch.from_numpy(a.view(np.uint8).reshape(rows, -1).copy())

    return cfg, get, lambda: None


def _fused_experts(i: str, kind: str, parts: dict[str, tuple]) -> dict[str, tuple]:
    """gpt-oss expert tensors of one layer as float32 [E, out, in] matrices and [E, out] biases
    under GGUF names.  MXFP4 (``_blocks`` + ``_scales``) is stored out-major already; the float form
    is [E, in, out] (multiplied from the right) and is transposed.  gate_up rows interleave the gate
    (even) and the linear branch (odd)."""
    out = {}
    if "_blocks" in parts:
        from . import mxfp4
        w = mxfp4.dequantize(parts["_blocks"][1], parts["_scales"][1])
    elif "" in parts:
        w = np.ascontiguousarray(np.swapaxes(_to_f32(*parts[""]), 1, 2))
    else:
        w = None
    b = _to_f32(*parts["_bias"]) if "_bias" in parts else None
    p = f"blk.{i}."
    if kind == "gate_up_proj":
        for nm, sl in (("ffn_gate_exps", slice(0, None, 2)), ("ffn_up_exps", slice(1, None, 2))):
            if w is not None:
                m = np.ascontiguousarray(w[:, sl])
                out[p + nm + ".weight"] = ("F32", m.shape, m)
            if b is not None:
                v = np.ascontiguousarray(b[:, sl])
                out[p + nm + ".bias"] = ("F32", v.shape, v)
    else:
        if w is not None:
            out[p + "ffn_down_exps.weight"] = ("F32", w.shape, np.ascontiguousarray(w))
        if b is not None:
            out[p + "ffn_down_exps.bias"] = ("F32", b.shape, np.ascontiguousarray(b))
    return out


def _dequant_rows(rows: np.ndarray, t: int, shape) -> np.ndarray:
    from ..gguf.quants import dequantize
    return dequantize(np.ascontiguousarray(rows).reshape(-1), t, shape).astype(np.float32).view(np.uint8).reshape(
        shape[0], -1)


def load_reference_tensors_hf(model_dir: str) -> tuple[ModelConfig, dict[str, torch.Tensor]]:
    """fp32 tensors under GGUF names for the reference model."""
    cfg, get, _ = hf_source(model_dir)
    from ..gguf.quants import dequantize
    out = {}
    names = ["token_embd.weight", "output_norm.weight"] + ([] if cfg.tie_embeddings else ["output.weight"])
    for i in range(cfg.n_layers):
        p = f"blk.{i}."
        if cfg.is_linear(i):
            names += [p + n for n in ("attn_norm.weight", "ffn_norm.weight", "ssm_in_qkv.weight", "ssm_in_z.weight",
                                      "ssm_in_b.weight", "ssm_in_a.weight", "ssm_conv1d.weight", "ssm_dt.bias",
                                      "ssm_a", "ssm_norm.weight", "ssm_out.weight", "ffn_gate.weight",
                                      "ffn_up.weight", "ffn_down.weight")]
            continue
        names += [p + n for n in ("attn_norm.weight", "ffn_norm.weight", "attn_q.weight", "attn_k.weight",
                                  "attn_v.weight", "attn_output.weight")]
        if cfg.qkv_bias:
            names += [p + n for n in ("attn_q.bias", "attn_k.bias", "attn_v.bias")]
        if cfg.attn_out_bias:
            names.append(p + "attn_output.bias")
        if cfg.attn_sinks:
            names.append(p + "attn_sinks.weight")
        if cfg.moe_bias:
            names += [p + n for n in ("ffn_gate_inp.bias", "ffn_gate_exps.bias", "ffn_up_exps.bias",
                                      "ffn_down_exps.bias")]
        if cfg.qk_norm:
            names += [p + "attn_q_norm.weight", p + "attn_k_norm.weight"]
        if cfg.sandwich_norms:
            names += [p + "post_attention_norm.weight", p + "post_ffw_norm.weight"]
        if cfg.is_moe:
            names += [p + n for n in ("ffn_gate_inp.weight", "ffn_gate_exps.weight", "ffn_up_exps.weight",
                                      "ffn_down_exps.weight")]
        else:
            names += [p + n for n in ("ffn_gate.weight", "ffn_up.weight", "ffn_down.weight")]
    for n in names:
        shape, t, raw = get(n)
        out[n] = torch.from_numpy(dequantize(raw.numpy().reshape(-1), t, shape).astype(np.float32))
    if cfg.tie_embeddings:
        out["output.weight"] = out["token_embd.weight"]
    return cfg, out
