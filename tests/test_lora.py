"""LoRA adapters (CPU): PEFT adapter files, dynamic deltas == merged weights, bundle switching and
composition, and logits against transformers running the patched weights."""
import json

import numpy as np
import pytest
import torch

from fak_b200.models.hf import write_safetensors
from fak_b200.models.lora import LoRAAdapter, LoRASet, load_peft_adapter, merged_source


def _write_adapter(path, modules, r, alpha, d_in, d_out, seed, rslora=False):
    path.mkdir(parents=True, exist_ok=True)
    g = torch.Generator().manual_seed(seed)
    t = {}
    for m in modules:
        t[f"base_model.model.{m}.lora_A.weight"] = torch.randn(r, d_in[m], generator=g) * 0.1
        t[f"base_model.model.{m}.lora_B.weight"] = torch.randn(d_out[m], r, generator=g) * 0.1
    write_safetensors(str(path / "adapter_model.safetensors"), t)
    (path / "adapter_config.json").write_text(json.dumps({"r": r, "lora_alpha": alpha, "peft_type": "LORA",
                                                          "use_rslora": rslora, "target_modules": ["q_proj"]}))
    return t


def test_adapter_math_and_sets():
    g = torch.Generator().manual_seed(0)
    A, B = torch.randn(4, 32, generator=g), torch.randn(16, 4, generator=g)
    a = LoRAAdapter("blk.0.attn_q.weight", A, B, alpha=8.0, bundle="x")
    x = torch.randn(3, 32, generator=g)
    assert torch.allclose(a.delta(x), x @ (2.0 * B @ A).T, atol=1e-5)
    assert a.overhead_fraction() == pytest.approx(4 * 48 / (32 * 16))
    s = LoRASet()
    s.add(a)
    s.add(LoRAAdapter("blk.0.attn_q.weight", A * 2, B, alpha=4.0, bundle="y"))
    with pytest.raises(ValueError):
        s.add(LoRAAdapter("blk.0.attn_q.weight", A, B, alpha=1.0, bundle="x"))
    w = torch.randn(16, 32, generator=g)
    both = s.merge_into("blk.0.attn_q.weight", w)
    assert torch.allclose(both, w + 2.0 * B @ A + 1.0 * B @ (A * 2), atol=1e-5)   # composition is additive
    s.deactivate("y")
    assert torch.allclose(s.merge_into("blk.0.attn_q.weight", w), w + 2.0 * B @ A, atol=1e-5)
    assert s.bundles() == ["x", "y"] and s.targets() == ["blk.0.attn_q.weight"]
    s.deactivate("x")
    assert s.delta("blk.0.attn_q.weight", x) is None
    with pytest.raises(ValueError):
        LoRAAdapter("t", torch.randn(4, 8), torch.randn(8, 3), 1.0)


def test_dynamic_equals_merged_on_the_reference_model(tmp_path):
    from fak_b200.config import preset
    from fak_b200.gguf.synth import write_synthetic_gguf
    from fak_b200.models.loader import load_reference_tensors
    from fak_b200.models.reference import ReferenceModel
    from fak_b200.models.weights import gguf_source
    from fak_b200.gguf.quants import dequantize
    cfg = preset("tiny-llama")
    path = str(tmp_path / "m.gguf")
    write_synthetic_gguf(path, cfg, "f32", seed=1, std=0.05)
    d, q, kv, f = cfg.d_model, cfg.q_dim, cfg.kv_dim, cfg.ffn_dim
    mods = ["model.layers.0.self_attn.q_proj", "model.layers.1.mlp.down_proj", "model.layers.0.self_attn.v_proj"]
    d_in = {mods[0]: d, mods[1]: f, mods[2]: d}
    d_out = {mods[0]: q, mods[1]: d, mods[2]: kv}
    _write_adapter(tmp_path / "ad", mods, 8, 16, d_in, d_out, seed=2)
    ls = load_peft_adapter(str(tmp_path / "ad"))
    assert ls.targets() == ["blk.0.attn_q.weight", "blk.0.attn_v.weight", "blk.1.ffn_down.weight"]
    _, tensors = load_reference_tensors(path)
    ids = torch.tensor([1, 5, 9, 200, 33])
    base = ReferenceModel(cfg, tensors).forward(ids)
    dyn_model = ReferenceModel(cfg, tensors)
    dyn_model.set_lora(ls)
    dyn = dyn_model.forward(ids)
    # merged through the device weight source (f32 blocks stay f32), read back as reference tensors
    _, get, _ = merged_source(gguf_source(path), ls)
    merged = dict(tensors)
    for n in ls.targets():
        shape, t, raw = get(n)
        merged[n] = torch.from_numpy(dequantize(raw.numpy().reshape(-1), t, shape))
    mer = ReferenceModel(cfg, merged).forward(ids)
    assert (dyn - base).abs().max() > 1e-2            # the adapter changes the model
    assert torch.allclose(dyn, mer, atol=2e-4, rtol=1e-4), (dyn - mer).abs().max()
    ls.deactivate("ad")
    assert torch.equal(dyn_model.forward(ids), base)  # switched off: the base model exactly


def test_lora_logits_match_transformers_patched_weights(tmp_path):
    transformers = pytest.importorskip("transformers")
    from fak_b200.models.hf import load_reference_tensors_hf
    from fak_b200.models.reference import ReferenceModel
    cfg = transformers.LlamaConfig(vocab_size=512, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                                   num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=256,
                                   rms_norm_eps=1e-6, tie_word_embeddings=False)
    torch.manual_seed(0)
    m = transformers.LlamaForCausalLM(cfg).eval().float()
    for p in m.parameters():
        torch.nn.init.normal_(p, std=0.05 if p.dim() > 1 else 0.5)
    mdir = tmp_path / "base"
    mdir.mkdir()
    write_safetensors(str(mdir / "model.safetensors"), dict(m.state_dict()))
    hf = m.config.to_dict()
    hf["architectures"] = ["LlamaForCausalLM"]
    (mdir / "config.json").write_text(json.dumps(hf))
    mods = ["model.layers.1.self_attn.k_proj", "model.layers.0.mlp.gate_proj"]
    t = _write_adapter(tmp_path / "ad", mods, 4, 8, {mods[0]: 128, mods[1]: 128}, {mods[0]: 64, mods[1]: 256},
                       seed=5, rslora=True)
    sd = m.state_dict()
    for mod in mods:   # PEFT semantics: W += alpha / sqrt(r) * B A with rsLoRA
        A, B = t[f"base_model.model.{mod}.lora_A.weight"], t[f"base_model.model.{mod}.lora_B.weight"]
        sd[mod + ".weight"].add_(8 / 2 * B @ A)
    ours_cfg, tensors = load_reference_tensors_hf(str(mdir))
    ref = ReferenceModel(ours_cfg, tensors)
    ref.set_lora(load_peft_adapter(str(tmp_path / "ad")))
    ids = torch.tensor([3, 17, 200, 45, 9])
    with torch.no_grad():
        want = m(ids[None]).logits[0]
    assert torch.allclose(ref.forward(ids), want, atol=2e-4, rtol=1e-4)
