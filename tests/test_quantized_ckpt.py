"""AWQ / GPTQ int4 checkpoints (CPU): packing round trips, the G4 device blocks, and end-to-end
logits of a quantized Llama checkpoint against transformers running the same dequantized weights."""
import json

import numpy as np
import pytest
import torch

from fak_b200.gguf import GGMLType
from fak_b200.gguf.quants import dequantize, quantize
from fak_b200.models import quantized_ckpt as qk


def _rand_quant(out_, in_, group, seed=0):
    rng = np.random.default_rng(seed)
    codes = rng.integers(0, 16, (out_, in_)).astype(np.uint8)
    s = (rng.random((out_, in_ // group)) * 0.01 + 1e-3).astype(np.float16).astype(np.float32)
    z = rng.integers(1, 16, (out_, in_ // group)).astype(np.float32)
    return codes, s, z


def test_awq_pack_order_and_roundtrip():
    codes, s, z = _rand_quant(64, 512, 128)
    qw, qz, sc = qk.pack_awq(codes, s, z)
    assert qw.shape == (512, 8) and qz.shape == (4, 8) and sc.dtype == np.float16
    word = int(qw[0, 0]) & 0xFFFFFFFF
    # nibble p holds logical output column AWQ_ORDER[p]
    assert [(word >> (4 * p)) & 15 for p in range(8)] == [int(codes[qk.AWQ_ORDER[p], 0]) for p in range(8)]
    c2, s2, z2, _ = qk.unpack_awq(qw, qz, sc, 128)
    assert (c2 == codes).all() and np.array_equal(s2, s) and np.array_equal(z2, z)


@pytest.mark.parametrize("v1", [True, False])
def test_gptq_roundtrip(v1):
    codes, s, z = _rand_quant(32, 256, 128, seed=1)
    qw, qz, sc = qk.pack_gptq(codes, s, z, 4, v1)
    assert qw.shape == (32, 32)
    c2, s2, z2, gi = qk.unpack_gptq(qw, qz, sc, None, 4, 128, v1)
    assert (c2 == codes).all() and np.array_equal(z2, z) and np.array_equal(gi, np.arange(256) // 128)


def test_g4_blocks_equal_dequantized_checkpoint():
    codes, s, z = _rand_quant(48, 768, 128, seed=2)
    rows, t = qk.device_rows(codes, s, z, np.arange(768) // 128, 128)
    assert t == GGMLType.G4 and rows.shape == (48, 3 * 144)
    got = dequantize(rows.reshape(-1), t, (48, 768))
    want = qk.dequant(codes, s, z, np.arange(768) // 128)
    np.testing.assert_allclose(got, want, rtol=1e-6, atol=1e-7)
    # groups of 256 map onto two equal 128-groups; act-order and 64-groups fall back to float32
    codes2, s2, z2 = _rand_quant(16, 512, 256, seed=3)
    rows2, t2 = qk.device_rows(codes2, s2, z2, np.arange(512) // 256, 256)
    np.testing.assert_allclose(dequantize(rows2.reshape(-1), t2, (16, 512)),
                               qk.dequant(codes2, s2, z2, np.arange(512) // 256), rtol=1e-6, atol=1e-7)
    perm = np.random.default_rng(0).permutation(np.arange(768) // 128)
    assert qk.device_rows(codes, s, z, perm, 128)[1] == GGMLType.F32
    c64, s64, z64 = _rand_quant(16, 512, 64)
    assert qk.device_rows(c64, s64, z64, np.arange(512) // 64, 64)[1] == GGMLType.F32


def test_g4_quantizer_error_bound():
    x = (np.random.default_rng(4).standard_normal((8, 1024)) * 0.05).astype(np.float32)
    y = dequantize(quantize(x, GGMLType.G4), GGMLType.G4, x.shape)
    g = x.reshape(-1, 128)
    step = (np.maximum(g.max(1), 0) - np.minimum(g.min(1), 0)) / 15
    assert (np.abs(x - y).reshape(-1, 128) <= step[:, None] * 0.5 + 1e-7).all()


def _rtn(w: np.ndarray, group: int):
    """Asymmetric round-to-nearest int4 per (output row, input group): codes, scales (f16-exact), zeros."""
    out_, in_ = w.shape
    g = w.reshape(out_, in_ // group, group)
    lo, hi = np.minimum(g.min(-1), 0), np.maximum(g.max(-1), 0)
    s = ((hi - lo) / 15).astype(np.float16).astype(np.float32)
    s = np.where(s > 0, s, 1).astype(np.float32)
    z = np.clip(np.rint(-lo / s), 0, 15).astype(np.float32)
    q = np.clip(np.rint(g / s[..., None]) + z[..., None], 0, 15).astype(np.uint8).reshape(out_, in_)
    return q, s, z


@pytest.mark.parametrize("method", ["awq", "gptq", "gptq_actorder"])
def test_quantized_llama_logits_match_transformers(method, tmp_path):
    transformers = pytest.importorskip("transformers")
    from fak_b200.models.hf import hf_source, load_reference_tensors_hf, write_safetensors
    from fak_b200.models.reference import ReferenceModel
    cfg = transformers.LlamaConfig(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                                   num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=256,
                                   rms_norm_eps=1e-6, tie_word_embeddings=False)
    torch.manual_seed(0)
    m = transformers.LlamaForCausalLM(cfg)
    for p in m.parameters():
        torch.nn.init.normal_(p, std=0.05 if p.dim() > 1 else 0.5)
    m = m.eval().float()
    tensors, group = {}, 128
    sd = m.state_dict()
    for name, w in sd.items():
        proj = name.endswith("_proj.weight") and ".layers." in name
        if not proj:
            tensors[name] = w
            continue
        base = name[: -len(".weight")]
        q, s, z = _rtn(w.numpy(), group)
        gidx = np.arange(w.shape[1]) // group
        if method == "gptq_actorder":   # inputs assigned to groups in a permuted order
            gidx = np.random.default_rng(len(name)).permutation(gidx)
            g = w.numpy()
            s = np.stack([((np.maximum(g[:, gidx == k].max(1), 0) - np.minimum(g[:, gidx == k].min(1), 0)) / 15)
                          for k in range(w.shape[1] // group)], 1).astype(np.float16).astype(np.float32)
            s = np.where(s > 0, s, 1).astype(np.float32)
            z = np.clip(np.rint(-np.stack([np.minimum(g[:, gidx == k].min(1), 0) for k in range(s.shape[1])], 1)
                                / s), 0, 15).astype(np.float32)
            q = np.clip(np.rint(g / s[:, gidx]) + z[:, gidx], 0, 15).astype(np.uint8)
        sd[name].copy_(torch.from_numpy(qk.dequant(q, s, z, gidx)))   # transformers runs the same weights
        if method == "awq":
            qw, qz, sc = qk.pack_awq(q, s, z)
        else:
            qw, qz, sc = qk.pack_gptq(q, s, z, 4, True)
            tensors[base + ".g_idx"] = torch.from_numpy(gidx.astype(np.int32))
        tensors[base + ".qweight"] = torch.from_numpy(qw)
        tensors[base + ".qzeros"] = torch.from_numpy(qz)
        tensors[base + ".scales"] = torch.from_numpy(sc)
    write_safetensors(str(tmp_path / "model.safetensors"), tensors)
    d = m.config.to_dict()
    d["architectures"] = ["LlamaForCausalLM"]
    d["quantization_config"] = ({"quant_method": "awq", "bits": 4, "group_size": group, "version": "gemm",
                                 "zero_point": True} if method == "awq" else
                                {"quant_method": "gptq", "bits": 4, "group_size": group,
                                 "desc_act": method == "gptq_actorder", "checkpoint_format": "gptq"})
    (tmp_path / "config.json").write_text(json.dumps(d))
    _, get, _ = hf_source(str(tmp_path))
    shape, t, _ = get("blk.0.attn_q.weight")
    assert shape == (256, 256) and t == (GGMLType.F32 if method == "gptq_actorder" else GGMLType.G4)
    ours_cfg, ref_t = load_reference_tensors_hf(str(tmp_path))
    ref = ReferenceModel(ours_cfg, ref_t)
    ids = torch.tensor([3, 17, 200, 45, 9, 311, 7])
    with torch.no_grad():
        want = m(ids[None]).logits[0]
    got = ref.forward(ids)
    assert torch.allclose(got, want, atol=3e-4, rtol=1e-4), (got - want).abs().max()


def test_g4_synthetic_gguf_loads_in_the_reference(tmp_path):
    from fak_b200.config import preset
    from fak_b200.gguf.synth import write_synthetic_gguf
    from fak_b200.models.loader import load_reference_tensors
    path = str(tmp_path / "g4.gguf")
    write_synthetic_gguf(path, preset("tiny-qwen2"), "g4", seed=1, std=0.05)
    from fak_b200.gguf import open_gguf
    types = {int(t.ggml_type) for t in open_gguf(path).tensors.values()}
    assert int(GGMLType.G4) in types and int(GGMLType.Q8_0) in types
    cfg, tensors = load_reference_tensors(path)
    assert tensors["blk.0.attn_q.weight"].shape == (cfg.q_dim, cfg.d_model)


def test_exl2_packing_roundtrip_and_error_bound():
    from fak_b200.models import exl2
    rng = np.random.default_rng(0)
    groups = [(4, 32), (3, 64), (8, 32), (2, 96), (5, 32), (6, 32)]
    in_ = sum(s for _, s in groups)
    codes = np.concatenate([rng.integers(0, 1 << b, (7, s)) for b, s in groups], axis=1)
    qw = exl2.pack(codes, groups)
    assert qw.dtype == np.int32 and qw.shape == (7, -(-sum(b * s for b, s in groups) // 32))
    assert (exl2.unpack(qw, groups) == codes).all()
    w = (rng.standard_normal((7, in_)) * 0.1).astype(np.float32)
    perm = rng.permutation(in_)
    t = exl2.quantize(w, groups, perm)
    d = exl2.dequantize(*t)
    scale = (t[2].astype(np.float32) * t[3].astype(np.float32)[None, :])
    bits, _, gidx, _ = exl2._bit_layout(groups)
    bound = np.empty_like(w)
    bound[:, perm] = scale[:, gidx] * 0.5 + 1e-6
    assert (np.abs(d - w) <= bound * 1.01).all()


def test_exl2_llama_logits_match_transformers(tmp_path):
    transformers = pytest.importorskip("transformers")
    from fak_b200.models import exl2
    from fak_b200.models.hf import load_reference_tensors_hf, write_safetensors
    from fak_b200.models.reference import ReferenceModel
    cfg = transformers.LlamaConfig(vocab_size=512, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                                   num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=256,
                                   rms_norm_eps=1e-6, tie_word_embeddings=False)
    torch.manual_seed(0)
    m = transformers.LlamaForCausalLM(cfg)
    for p in m.parameters():
        torch.nn.init.normal_(p, std=0.05 if p.dim() > 1 else 0.5)
    m = m.eval().float()
    sd = m.state_dict()
    tensors = {}
    rng = np.random.default_rng(1)
    for name, w in sd.items():
        if not (name.endswith("_proj.weight") and ".layers." in name):
            tensors[name] = w
            continue
        in_ = w.shape[1]
        groups = [(6, in_ // 4), (4, in_ // 2), (3, in_ // 4)]
        qw, qg, qs, qm, qi = exl2.quantize(w.numpy(), groups, rng.permutation(in_))
        sd[name].copy_(torch.from_numpy(exl2.dequantize(qw, qg, qs, qm, qi)))
        base = name[: -len(".weight")]
        tensors[base + ".q_weight"] = torch.from_numpy(qw)
        tensors[base + ".q_groups"] = torch.from_numpy(qg.astype(np.int32)).to(torch.int32)
        tensors[base + ".q_scale"] = torch.from_numpy(qs)
        tensors[base + ".q_scale_max"] = torch.from_numpy(qm)
        tensors[base + ".q_invperm"] = torch.from_numpy(qi)
    write_safetensors(str(tmp_path / "model.safetensors"), tensors)
    d = m.config.to_dict()
    d["architectures"] = ["LlamaForCausalLM"]
    d["quantization_config"] = {"quant_method": "exl2", "bits": 4.5}
    (tmp_path / "config.json").write_text(json.dumps(d))
    ours_cfg, ref_t = load_reference_tensors_hf(str(tmp_path))
    ids = torch.tensor([3, 17, 200, 45, 9, 311, 7])
    with torch.no_grad():
        want = m(ids[None]).logits[0]
    got = ReferenceModel(ours_cfg, ref_t).forward(ids)
    assert torch.allclose(got, want, atol=3e-4, rtol=1e-4), (got - want).abs().max()
