"""Hugging Face checkpoints (safetensors + config.json): our fp32 reference model, loaded through
the HF source, reproduces the transformers implementation's logits (CPU)."""
import json

import pytest
import torch

transformers = pytest.importorskip("transformers")

from fak_b200.models.hf import config_from_hf, hf_source, load_reference_tensors_hf, read_safetensors, write_safetensors  # noqa: E402
from fak_b200.models.reference import ReferenceModel  # noqa: E402


def _save(model, tmp_path):
    write_safetensors(str(tmp_path / "model.safetensors"), {k: v for k, v in model.state_dict().items()})
    cfg = model.config.to_dict()
    cfg["architectures"] = [type(model).__name__]
    (tmp_path / "config.json").write_text(json.dumps(cfg))
    return str(tmp_path)


@pytest.mark.parametrize("arch", ["qwen2", "llama", "qwen3"])
def test_reference_matches_transformers(arch, tmp_path):
    common = dict(vocab_size=512, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                  num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=256, rms_norm_eps=1e-6,
                  rope_theta=10000.0, tie_word_embeddings=False)
    if arch == "qwen2":
        m = transformers.Qwen2ForCausalLM(transformers.Qwen2Config(**common))
    elif arch == "llama":
        m = transformers.LlamaForCausalLM(transformers.LlamaConfig(**common, attention_bias=False, mlp_bias=False))
    else:
        m = transformers.Qwen3ForCausalLM(transformers.Qwen3Config(**common, head_dim=32))
    torch.manual_seed(0)
    for p in m.parameters():  # visible norms / biases
        torch.nn.init.normal_(p, std=0.05 if p.dim() > 1 else 0.5)
    m = m.eval().float()
    d = _save(m, tmp_path)
    cfg, tensors = load_reference_tensors_hf(d)
    assert cfg.arch == arch and cfg.n_kv_heads == 2
    ref = ReferenceModel(cfg, tensors)
    ids = torch.tensor([3, 17, 200, 45, 9, 311, 7])
    with torch.no_grad():
        want = m(ids[None]).logits[0]
    got = ref.forward(ids)
    assert torch.allclose(got, want, atol=2e-4, rtol=1e-4), (got - want).abs().max()


def test_safetensors_roundtrip_and_bf16(tmp_path):
    t = {"a": torch.randn(3, 5), "b": torch.randn(4).bfloat16(), "c": torch.randn(2, 2).half()}
    write_safetensors(str(tmp_path / "x.safetensors"), t, {"format": "pt"})
    r = read_safetensors(str(tmp_path / "x.safetensors"))
    assert r["a"][0] == "F32" and torch.equal(torch.from_numpy(r["a"][2].copy()), t["a"])
    assert r["b"][0] == "BF16" and torch.equal(torch.from_numpy(r["b"][2].copy()).view(torch.bfloat16), t["b"])
    assert r["c"][1] == (2, 2)


def test_hf_source_feeds_the_device_loader_shapes(tmp_path):
    m = transformers.Qwen2ForCausalLM(transformers.Qwen2Config(
        vocab_size=256, hidden_size=64, intermediate_size=128, num_hidden_layers=1, num_attention_heads=2,
        num_key_value_heads=1, tie_word_embeddings=True))
    d = _save(m.eval(), tmp_path)
    cfg, get, close = hf_source(d)
    assert cfg.tie_embeddings and cfg.qkv_bias
    shape, t, raw = get("blk.0.attn_q.weight")
    assert shape == (64, 64) and raw.shape == (64, 64 * 4)
    with pytest.raises(ValueError):
        config_from_hf({"architectures": ["GPT2LMHeadModel"], "hidden_size": 8, "num_attention_heads": 2,
                        "num_hidden_layers": 1, "vocab_size": 10})


@pytest.mark.parametrize("longrope", [False, True])
def test_phi3_fused_projections_and_longrope(longrope, tmp_path):
    """Phi-3: fused qkv / gate_up projections split on load; longrope factors pinned to the
    model's max-context regime."""
    kw = dict(vocab_size=512, hidden_size=128, intermediate_size=256, num_hidden_layers=2, num_attention_heads=4,
              num_key_value_heads=2, max_position_embeddings=512, pad_token_id=0, bos_token_id=1, eos_token_id=2,
              rms_norm_eps=1e-5, tie_word_embeddings=False)
    if longrope:
        kw["original_max_position_embeddings"] = 128
        kw["rope_parameters"] = {"rope_type": "longrope", "rope_theta": 10000.0,
                                 "short_factor": [1.0 + 0.02 * i for i in range(16)],
                                 "long_factor": [1.0 + 0.3 * i for i in range(16)]}
    m = transformers.Phi3ForCausalLM(transformers.Phi3Config(**kw))
    torch.manual_seed(0)
    for p in m.parameters():
        torch.nn.init.normal_(p, std=0.05 if p.dim() > 1 else 0.5)
    m = m.eval().float()
    d = _save(m, tmp_path)
    cfg, tensors = load_reference_tensors_hf(d)
    assert cfg.arch == "llama" and tensors["blk.0.attn_k.weight"].shape == (64, 128)
    if longrope:
        assert dict(cfg.rope_scaling)["original_max_position_embeddings"] == 128
    ref = ReferenceModel(cfg, tensors)
    ids = torch.tensor([3, 17, 200, 45, 9, 311, 7, 99])
    with torch.no_grad():
        # transformers switches longrope factors by the live length; our tables pin the long factor
        # (the model's max context exceeds the original), which transformers uses past 128 tokens
        want = m(ids[None]).logits[0] if not longrope else None
    got = ref.forward(ids)
    if not longrope:
        assert torch.allclose(got, want, atol=2e-4, rtol=1e-4), (got - want).abs().max()
    else:
        long_ids = torch.randint(0, 512, (140,), generator=torch.Generator().manual_seed(1))
        with torch.no_grad():
            want_long = m(long_ids[None]).logits[0]
        assert torch.allclose(ref.forward(long_ids), want_long, atol=3e-4, rtol=1e-4)


def test_gemma2_matches_transformers(tmp_path):
    """Gemma-2: GELU-tanh gated FFN, sandwich norms with (1 + w) scales, score and final-logit
    soft-capping, query_pre_attn_scalar, embedding scale, alternating sliding windows."""
    c = transformers.Gemma2Config(vocab_size=512, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                                  num_attention_heads=4, num_key_value_heads=2, head_dim=32,
                                  max_position_embeddings=512, pad_token_id=0, bos_token_id=2, eos_token_id=1,
                                  sliding_window=6, query_pre_attn_scalar=24, attn_logit_softcapping=5.0,
                                  final_logit_softcapping=3.0)
    m = transformers.Gemma2ForCausalLM(c)
    m.config._attn_implementation = "eager"
    torch.manual_seed(0)
    for p in m.parameters():
        torch.nn.init.normal_(p, std=0.08 if p.dim() > 1 else 0.3)
    m = m.eval().float()
    d = _save(m, tmp_path)
    cfg, tensors = load_reference_tensors_hf(d)
    assert cfg.arch == "gemma2" and cfg.sandwich_norms and cfg.act == "gelu_tanh"
    assert [cfg.layer_window(i) for i in range(2)] == [6, 0]
    ref = ReferenceModel(cfg, tensors)
    ids = torch.tensor([3, 17, 200, 45, 9, 311, 7, 99, 12, 400, 5])
    with torch.no_grad():
        want = m(ids[None]).logits[0]
    got = ref.forward(ids)
    assert torch.allclose(got, want, atol=2e-4, rtol=1e-4), (got - want).abs().max()
