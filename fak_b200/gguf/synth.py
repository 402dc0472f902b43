"""Random-init checkpoints of a named architecture, written as GGUF.

Weights are N(0, std) (std 0.02 by default), norm gains are 1, and every
tensor is generated from its own seeded stream so a tensor's values do not
depend on which other tensors were generated.  The quantization mix follows
llama.cpp's naming conventions:

* ``q8_0``   -- every 2-D weight Q8_0, norms/router f32.
* ``q4_k_m`` -- Q4_K everywhere except ``output.weight`` (Q6_K) and the
  ``attn_v`` / ``ffn_down`` weights of layers picked by ``use_more_bits``
  (Q6_K), which is how llama.cpp's Q4_K_M recipe spends extra bits.
* ``g4``     -- AWQ / GPTQ-style int4 (G4 blocks, groups of 128) for the layer matrices, Q8_0
  embeddings and LM head.
* ``f32`` / ``f16`` / ``bf16`` -- unquantized.

Rows whose length is not a multiple of 256 cannot hold K-quant blocks and fall
back to Q8_0.  The reference builds its fixtures the same way (seeded synthetic
weights, internal/model/synthetic.go:9-60) but in-process; here the fixture is
an on-disk GGUF so the loader path is exercised end to end.

With ``device="cuda"`` the values are generated and quantized on the GPU by
the framework's own quantize kernels, which is what makes multi-GB benchmark
checkpoints practical to build on the fly.
"""
from __future__ import annotations

import hashlib
from typing import Callable, Iterator

import numpy as np

from ..config import ModelConfig
from .constants import (FILE_TYPE_ALL_F32, FILE_TYPE_MOSTLY_BF16, FILE_TYPE_MOSTLY_F16, FILE_TYPE_MOSTLY_Q4_K_M,
                        FILE_TYPE_MOSTLY_Q8_0, GGMLType, QK_K, ValueType)
from .quants import quantize
from .writer import GGUFWriter

QUANT_MIXES = ("q8_0", "q4_k_m", "g4", "f32", "f16", "bf16")


def use_more_bits(i: int, n: int) -> bool:
    """llama.cpp's Q4_K_M layer selector for the attn_v / ffn_down upgrade to Q6_K."""
    return i < n // 8 or i >= 7 * n // 8 or (i - n // 8) % 3 == 2


def tensor_plan(cfg: ModelConfig) -> list[tuple[str, tuple[int, ...], str]]:
    """(gguf name, numpy shape, role) for every tensor of the architecture."""
    d, L = cfg.d_model, cfg.n_layers
    out: list[tuple[str, tuple[int, ...], str]] = [("token_embd.weight", (cfg.vocab_size, d), "embed")]
    for i in range(L):
        p = f"blk.{i}."
        out.append((p + "attn_norm.weight", (d,), "norm"))
        out.append((p + "attn_q.weight", (cfg.q_dim, d), "attn_q"))
        out.append((p + "attn_k.weight", (cfg.kv_dim, d), "attn_k"))
        out.append((p + "attn_v.weight", (cfg.kv_dim, d), "attn_v"))
        if cfg.qkv_bias:
            out.append((p + "attn_q.bias", (cfg.q_dim,), "bias"))
            out.append((p + "attn_k.bias", (cfg.kv_dim,), "bias"))
            out.append((p + "attn_v.bias", (cfg.kv_dim,), "bias"))
        if cfg.qk_norm:
            out.append((p + "attn_q_norm.weight", (cfg.head_dim,), "norm"))
            out.append((p + "attn_k_norm.weight", (cfg.head_dim,), "norm"))
        out.append((p + "attn_output.weight", (d, cfg.q_dim), "attn_output"))
        out.append((p + "ffn_norm.weight", (d,), "norm"))
        if cfg.sandwich_norms:
            out.append((p + "post_attention_norm.weight", (d,), "norm"))
            out.append((p + "post_ffw_norm.weight", (d,), "norm"))
        if cfg.is_moe:
            E, f = cfg.n_experts, cfg.expert_ffn_dim
            out.append((p + "ffn_gate_inp.weight", (E, d), "router"))
            out.append((p + "ffn_gate_exps.weight", (E, f, d), "ffn_gate"))
            out.append((p + "ffn_up_exps.weight", (E, f, d), "ffn_up"))
            out.append((p + "ffn_down_exps.weight", (E, d, f), "ffn_down"))
        else:
            out.append((p + "ffn_gate.weight", (cfg.ffn_dim, d), "ffn_gate"))
            out.append((p + "ffn_up.weight", (cfg.ffn_dim, d), "ffn_up"))
            out.append((p + "ffn_down.weight", (d, cfg.ffn_dim), "ffn_down"))
    out.append(("output_norm.weight", (d,), "norm"))
    if not cfg.tie_embeddings:
        out.append(("output.weight", (cfg.vocab_size, d), "output"))
    return out


def _layer_of(name: str) -> int:
    return int(name.split(".")[1]) if name.startswith("blk.") else -1


def choose_type(cfg: ModelConfig, name: str, shape: tuple[int, ...], role: str, mix: str) -> GGMLType:
    if role in ("norm", "bias", "router") or len(shape) == 1:
        return GGMLType.F32
    if mix == "f32":
        return GGMLType.F32
    if mix == "f16":
        return GGMLType.F16
    if mix == "bf16":
        return GGMLType.BF16
    row = shape[-1]
    if mix == "q8_0":
        return GGMLType.Q8_0 if row % 32 == 0 else GGMLType.F16
    if mix == "q4_k_m":
        if row % QK_K:
            return GGMLType.Q8_0 if row % 32 == 0 else GGMLType.F16
        if role == "output":
            return GGMLType.Q6_K
        if role in ("attn_v", "ffn_down") and use_more_bits(_layer_of(name), cfg.n_layers):
            return GGMLType.Q6_K
        return GGMLType.Q4_K
    if mix == "g4":  # AWQ / GPTQ-style checkpoints: int4 groups of 128 for the block matrices
        if role in ("embed", "output") or row % QK_K:
            return GGMLType.Q8_0 if row % 32 == 0 else GGMLType.F16
        return GGMLType.G4
    raise ValueError(f"unknown quant mix {mix!r}; choose one of {QUANT_MIXES}")


def _seed_for(seed: int, name: str) -> int:
    h = hashlib.blake2b(f"{seed}:{name}".encode(), digest_size=8).digest()
    return int.from_bytes(h, "little") & 0x7FFFFFFFFFFFFFFF


def init_values_cpu(name: str, shape: tuple[int, ...], role: str, seed: int, std: float) -> np.ndarray:
    if role == "norm":
        return np.ones(shape, np.float32)
    rng = np.random.default_rng(_seed_for(seed, name))
    return (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)


def synth_tensors(cfg: ModelConfig, mix: str = "q8_0", seed: int = 0, std: float = 0.02, device: str = "cpu"
                  ) -> Iterator[tuple[str, tuple[int, ...], GGMLType, Callable[[], np.ndarray]]]:
    """Yield (name, shape, type, payload-thunk) for every tensor; payloads are GGML bytes."""
    for name, shape, role in tensor_plan(cfg):
        t = choose_type(cfg, name, shape, role, mix)

        def thunk(name=name, shape=shape, role=role, t=t) -> np.ndarray:
            if device == "cpu" or t in (GGMLType.F32, GGMLType.F16, GGMLType.BF16) and role == "norm":
                return quantize(init_values_cpu(name, shape, role, seed, std), t)
            from ..ops import quant as dq
            return dq.synth_quantized(shape, t, _seed_for(seed, name), std, ones=(role == "norm")).cpu().numpy()

        yield name, shape, t, thunk


def synthetic_vocab(cfg: ModelConfig) -> tuple[list[str], list[int], list[str]]:
    """A byte-level BPE vocabulary of exactly ``cfg.vocab_size`` entries.

    Ids ``bos/eos`` (and their neighbours used by ChatML) carry the special
    tokens; 256 byte tokens use GPT-2's byte-to-unicode alphabet; a block of
    lowercase-pair merges makes the BPE do real work; the remainder are unused
    placeholder tokens.
    """
    from ..tokenizer.bpe import bytes_to_unicode
    V = cfg.vocab_size
    tokens: list[str | None] = [None] * V
    types = [1] * V
    specials = {"<|endoftext|>": None, "<|im_start|>": None, "<|im_end|>": None}
    if cfg.eos_token_id >= 3 and cfg.eos_token_id < V:
        base = cfg.eos_token_id - 2
    else:
        base = 0
    for k, name in enumerate(specials):
        tokens[base + k] = name
        types[base + k] = 3
    b2u = bytes_to_unicode()
    free = (i for i in range(V) if tokens[i] is None)
    for b in range(256):
        i = next(free)
        tokens[i] = b2u[b]
    letters = "abcdefghijklmnopqrstuvwxyz"
    merges: list[str] = []
    sp = b2u[ord(" ")]
    for a in letters:
        for c in letters:
            if len(merges) >= max(0, V - 300):
                break
            merges.append(f"{a} {c}")
    for a in letters:
        merges.append(f"{sp} {a}")
    merges = merges[: max(0, V - 300)]
    have = set(t for t in tokens if t is not None)
    for m in merges:
        tok = m.replace(" ", "")
        if tok in have:
            continue
        try:
            i = next(free)
        except StopIteration:
            break
        tokens[i] = tok
        have.add(tok)
    n = 0
    for i in range(V):
        if tokens[i] is None:
            tokens[i] = f"<|unused_{n}|>"
            types[i] = 5
            n += 1
    return tokens, types, merges  # type: ignore[return-value]


_FILE_TYPE = {"q8_0": FILE_TYPE_MOSTLY_Q8_0, "q4_k_m": FILE_TYPE_MOSTLY_Q4_K_M, "f32": FILE_TYPE_ALL_F32,
              "f16": FILE_TYPE_MOSTLY_F16, "bf16": FILE_TYPE_MOSTLY_BF16,
              "g4": 1024}   # no llama.cpp file type holds G4 blocks: 1024 is llama.cpp's "guessed"


def write_metadata(w: GGUFWriter, cfg: ModelConfig, mix: str, with_vocab: bool = True) -> None:
    a = cfg.arch
    w.add("general.name", cfg.name or f"synthetic-{a}")
    w.add("general.file_type", _FILE_TYPE[mix], ValueType.UINT32)
    w.add("general.quantization_version", 2, ValueType.UINT32)
    w.add(f"{a}.block_count", cfg.n_layers, ValueType.UINT32)
    w.add(f"{a}.context_length", cfg.max_context, ValueType.UINT32)
    w.add(f"{a}.embedding_length", cfg.d_model, ValueType.UINT32)
    w.add(f"{a}.feed_forward_length", cfg.ffn_dim, ValueType.UINT32)
    w.add(f"{a}.attention.head_count", cfg.n_heads, ValueType.UINT32)
    w.add(f"{a}.attention.head_count_kv", cfg.n_kv_heads, ValueType.UINT32)
    w.add(f"{a}.attention.key_length", cfg.head_dim, ValueType.UINT32)
    w.add(f"{a}.attention.value_length", cfg.head_dim, ValueType.UINT32)
    w.add(f"{a}.attention.layer_norm_rms_epsilon", float(cfg.rms_eps), ValueType.FLOAT32)
    w.add(f"{a}.rope.freq_base", float(cfg.rope_theta), ValueType.FLOAT32)
    if cfg.sliding_window > 0 and (cfg.swa_layers is None or a == "gemma2"):   # every (gemma2: every other) layer
        w.add(f"{a}.attention.sliding_window", int(cfg.sliding_window), ValueType.UINT32)
    if a == "gemma2":
        w.add(f"{a}.attn_logit_softcapping", float(cfg.attn_softcap), ValueType.FLOAT32)
        w.add(f"{a}.final_logit_softcapping", float(cfg.final_softcap), ValueType.FLOAT32)
    if cfg.rope_scaling:
        rs = dict(cfg.rope_scaling)
        w.add(f"{a}.rope.scaling.type", str(rs.get("type") or rs.get("rope_type")))
        w.add(f"{a}.rope.scaling.factor", float(rs.get("factor", 1.0)), ValueType.FLOAT32)
        if "original_max_position_embeddings" in rs:
            w.add(f"{a}.rope.scaling.original_context_length", int(rs["original_max_position_embeddings"]),
                  ValueType.UINT32)
    w.add(f"{a}.vocab_size", cfg.vocab_size, ValueType.UINT32)
    if cfg.is_moe:
        w.add(f"{a}.expert_count", cfg.n_experts, ValueType.UINT32)
        w.add(f"{a}.expert_used_count", cfg.n_experts_used, ValueType.UINT32)
        w.add(f"{a}.expert_feed_forward_length", cfg.expert_ffn_dim, ValueType.UINT32)
        w.add(f"{a}.expert_weights_norm", bool(cfg.norm_topk_prob), ValueType.BOOL)
    w.add("tokenizer.ggml.bos_token_id", cfg.bos_token_id, ValueType.UINT32)
    w.add("tokenizer.ggml.eos_token_id", cfg.eos_token_id, ValueType.UINT32)
    if with_vocab:
        tokens, types, merges = synthetic_vocab(cfg)
        w.add("tokenizer.ggml.model", "gpt2")
        w.add("tokenizer.ggml.tokens", tokens, ValueType.ARRAY, ValueType.STRING)
        w.add("tokenizer.ggml.token_type", types, ValueType.ARRAY, ValueType.INT32)
        w.add("tokenizer.ggml.merges", merges, ValueType.ARRAY, ValueType.STRING)


def llama_rope_permute_rows(raw_rows: np.ndarray, n_heads: int, head_dim: int) -> np.ndarray:
    """Row order GGML's "llama" arch stores Q/K in (interleaved rotary pairs).

    HF order within a head is [first half | second half]; llama.cpp's converter
    interleaves them so pair j sits at rows (2j, 2j+1).  Rows are whole
    quantized rows, so this works on block bytes as well as on floats.
    """
    half = head_dim // 2
    r = raw_rows.reshape(n_heads, 2, half, -1)
    return np.ascontiguousarray(r.transpose(0, 2, 1, 3)).reshape(raw_rows.shape)


def write_synthetic_gguf(path: str, cfg: ModelConfig, mix: str = "q8_0", seed: int = 0, std: float = 0.02,
                         device: str = "cpu") -> str:
    cfg.validate()
    w = GGUFWriter(path, arch=cfg.arch)
    write_metadata(w, cfg, mix)
    for name, shape, t, thunk in synth_tensors(cfg, mix, seed, std, device):
        if cfg.arch == "llama" and (name.endswith("attn_q.weight") or name.endswith("attn_k.weight")):
            heads = cfg.n_heads if name.endswith("attn_q.weight") else cfg.n_kv_heads

            def permuted(thunk=thunk, shape=shape, heads=heads) -> np.ndarray:
                rows = thunk().reshape(shape[0], -1)
                return llama_rope_permute_rows(rows, heads, cfg.head_dim)
            w.add_tensor(name, shape, t, permuted)
        else:
            w.add_tensor(name, shape, t, thunk)
    w.write()
    return path
