"""Sliding-window attention (CPU): config parsing (Mistral / Qwen2 / layer_types / GGUF) and the
reference model's window mask against transformers."""
import json

import pytest
import torch

from fak_b200.config import ModelConfig, config_from_gguf_metadata
from fak_b200.models.hf import config_from_hf


def test_window_config_parsing():
    base = {"architectures": ["MistralForCausalLM"], "hidden_size": 64, "num_attention_heads": 2,
            "num_hidden_layers": 4, "vocab_size": 100}
    c = config_from_hf(dict(base, sliding_window=4096))
    assert [c.layer_window(i) for i in range(4)] == [4096] * 4 and c.max_window() == 4096
    q = config_from_hf(dict(base, architectures=["Qwen2ForCausalLM"], sliding_window=128, use_sliding_window=True,
                            max_window_layers=2))
    assert [q.layer_window(i) for i in range(4)] == [0, 0, 128, 128] and q.max_window() == 0
    assert config_from_hf(dict(base, architectures=["Qwen2ForCausalLM"], sliding_window=128,
                               use_sliding_window=False)).sliding_window == 0
    t = config_from_hf(dict(base, sliding_window=8, layer_types=["sliding_attention", "full_attention"] * 2))
    assert [t.layer_window(i) for i in range(4)] == [8, 0, 8, 0]
    hash(t)
    meta = {"general.architecture": "llama", "llama.block_count": 2, "llama.embedding_length": 128,
            "llama.attention.head_count": 4, "llama.attention.head_count_kv": 2, "llama.feed_forward_length": 256,
            "llama.vocab_size": 512, "llama.attention.sliding_window": 64}
    assert config_from_gguf_metadata(meta).max_window() == 64
    assert ModelConfig("llama", 2, 64, 2, 2, 32, 128, 100).max_window() == 0


@pytest.mark.parametrize("arch", ["mistral", "qwen2"])
def test_reference_window_matches_transformers(arch, tmp_path):
    transformers = pytest.importorskip("transformers")
    from fak_b200.models.hf import load_reference_tensors_hf, write_safetensors
    from fak_b200.models.reference import ReferenceModel
    common = dict(vocab_size=512, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                  num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=256, rms_norm_eps=1e-6,
                  rope_theta=10000.0, tie_word_embeddings=False, sliding_window=5)
    if arch == "mistral":
        m = transformers.MistralForCausalLM(transformers.MistralConfig(**common))
    else:
        m = transformers.Qwen2ForCausalLM(transformers.Qwen2Config(**common, use_sliding_window=True,
                                                                   max_window_layers=1))
    m.config._attn_implementation = "eager"
    torch.manual_seed(0)
    for p in m.parameters():
        torch.nn.init.normal_(p, std=0.05 if p.dim() > 1 else 0.5)
    m = m.eval().float()
    write_safetensors(str(tmp_path / "model.safetensors"), dict(m.state_dict()))
    d = m.config.to_dict()
    d["architectures"] = [type(m).__name__]
    (tmp_path / "config.json").write_text(json.dumps(d))
    cfg, tensors = load_reference_tensors_hf(str(tmp_path))
    assert cfg.layer_window(1) == 5 and cfg.layer_window(0) == (5 if arch == "mistral" else 0)
    ref = ReferenceModel(cfg, tensors)
    ids = torch.tensor([3, 17, 200, 45, 9, 311, 7, 100, 250, 11, 64, 2])
    with torch.no_grad():
        want = m(ids[None]).logits[0]
    got = ref.forward(ids)
    assert torch.allclose(got, want, atol=2e-4, rtol=1e-4), (got - want).abs().max()
    full = ReferenceModel(cfg.replace(sliding_window=0), tensors).forward(ids)
    assert (full[-1] - got[-1]).abs().max() > 1e-3      # the window changes late positions
    assert torch.allclose(full[:5], got[:5], atol=1e-5)  # but not those inside the first window


def test_gguf_roundtrip_of_window_and_rope_scaling(tmp_path):
    from fak_b200.config import preset
    from fak_b200.gguf.synth import write_synthetic_gguf
    from fak_b200.models.loader import open_model
    cfg = preset("tiny-llama").replace(sliding_window=32, rope_scaling={"type": "linear", "factor": 2.0})
    path = str(tmp_path / "m.gguf")
    write_synthetic_gguf(path, cfg, "q8_0", seed=0)
    _, c2 = open_model(path)
    assert c2.max_window() == 32 and dict(c2.rope_scaling) == {"type": "linear", "factor": 2.0}


def test_gemma2_gguf_roundtrip_and_reference_features(tmp_path):
    import torch
    from fak_b200.config import preset
    from fak_b200.gguf.synth import write_synthetic_gguf
    from fak_b200.models.reference import ReferenceModel
    cfg = preset("tiny-gemma2")
    path = str(tmp_path / "g.gguf")
    write_synthetic_gguf(path, cfg, "q8_0", seed=1, std=0.05)
    ref = ReferenceModel.from_gguf(path)
    c = ref.cfg
    assert (c.arch, c.act, c.sandwich_norms, c.attn_softcap, c.final_softcap) == ("gemma2", "gelu_tanh", True, 50.0, 30.0)
    assert c.embed_scale == 16.0 and [c.layer_window(i) for i in range(2)] == [32, 0]
    assert "blk.1.post_ffw_norm.weight" in ref.t
    logits = ref.forward(torch.arange(40))
    assert logits.abs().max() <= 30.0 + 1e-4          # final soft-cap
