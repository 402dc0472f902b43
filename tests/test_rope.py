"""Scaled RoPE (linear, llama3, yarn, longrope, dynamic): inverse frequencies and attention factor
against the transformers implementation, end-to-end logits of a rope-scaled Llama checkpoint, and
the GGUF ``rope.scaling.*`` keys (CPU)."""
import json

import pytest
import torch

from fak_b200.config import ModelConfig, config_from_gguf_metadata
from fak_b200.models.rope import cos_sin, inv_freq

transformers = pytest.importorskip("transformers")
from transformers.modeling_rope_utils import ROPE_INIT_FUNCTIONS  # noqa: E402

HD, THETA, MAXPOS = 64, 10000.0, 8192

CASES = [
    {"rope_type": "linear", "factor": 4.0},
    {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
     "original_max_position_embeddings": 1024},
    {"rope_type": "yarn", "factor": 4.0, "original_max_position_embeddings": 2048},
    {"rope_type": "yarn", "factor": 8.0, "original_max_position_embeddings": 1024, "beta_fast": 16, "beta_slow": 2,
     "mscale": 1.0, "mscale_all_dim": 0.5},
    {"rope_type": "yarn", "factor": 4.0, "original_max_position_embeddings": 2048, "truncate": False},
    {"rope_type": "longrope", "original_max_position_embeddings": 2048,
     "long_factor": [1.0 + 0.1 * i for i in range(HD // 2)], "short_factor": [1.0 + 0.01 * i for i in range(HD // 2)]},
]


def _hf_cfg(params):
    rp = dict(params, rope_theta=THETA)
    return transformers.LlamaConfig(hidden_size=HD * 4, num_attention_heads=4, max_position_embeddings=MAXPOS,
                                    rope_parameters=rp)


@pytest.mark.parametrize("params", CASES, ids=lambda p: p["rope_type"] + ("_ms" if "mscale" in p else "")
                         + ("_notrunc" if "truncate" in p else ""))
def test_inv_freq_matches_transformers(params):
    # longrope: the factor is pinned to the model's max-context regime (long past the original window)
    kw = {"seq_len": MAXPOS} if params["rope_type"] == "longrope" else {}
    want, want_att = ROPE_INIT_FUNCTIONS[params["rope_type"]](_hf_cfg(params), "cpu", **kw)
    got, att = inv_freq(HD, THETA, params, MAXPOS)
    assert torch.allclose(got.float(), want.float(), rtol=1e-6, atol=1e-9), (got, want)
    assert att == pytest.approx(float(want_att), rel=1e-6)


def test_config_hashable_and_cos_sin_scale():
    cfg = ModelConfig("llama", 2, 128, 4, 2, 32, 256, 512, rope_scaling={"type": "yarn", "factor": 4.0,
                                                                         "original_max_position_embeddings": 64})
    hash(cfg)
    assert dict(cfg.rope_scaling)["factor"] == 4.0
    c, s = cos_sin(torch.arange(4), 32, 1e4, cfg.rope_scaling)
    m = 0.1 * torch.log(torch.tensor(4.0)) + 1
    assert torch.allclose(c[0], torch.full((16,), float(m)))
    c0, _ = cos_sin(torch.arange(4), 32, 1e4, None)
    assert torch.equal(c0[0], torch.ones(16))


def test_gguf_rope_scaling_keys():
    meta = {"general.architecture": "llama", "llama.block_count": 2, "llama.embedding_length": 128,
            "llama.attention.head_count": 4, "llama.attention.head_count_kv": 2, "llama.feed_forward_length": 256,
            "llama.vocab_size": 512, "llama.rope.scaling.type": "yarn", "llama.rope.scaling.factor": 4.0,
            "llama.rope.scaling.original_context_length": 32768, "llama.rope.scaling.yarn_beta_fast": 32.0}
    cfg = config_from_gguf_metadata(meta)
    rs = dict(cfg.rope_scaling)
    assert rs == {"type": "yarn", "factor": 4.0, "original_max_position_embeddings": 32768, "beta_fast": 32.0}
    meta["llama.rope.scaling.type"] = "none"
    assert config_from_gguf_metadata(meta).rope_scaling is None


@pytest.mark.parametrize("params", [CASES[1], CASES[2]], ids=["llama3", "yarn"])
def test_scaled_llama_logits_match_transformers(params, tmp_path):
    from fak_b200.models.hf import load_reference_tensors_hf, write_safetensors
    from fak_b200.models.reference import ReferenceModel
    cfg = transformers.LlamaConfig(vocab_size=512, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                                   num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=MAXPOS,
                                   rms_norm_eps=1e-6, tie_word_embeddings=False,
                                   rope_parameters=dict(params, rope_theta=THETA))
    m = transformers.LlamaForCausalLM(cfg)
    torch.manual_seed(0)
    for p in m.parameters():
        torch.nn.init.normal_(p, std=0.05 if p.dim() > 1 else 0.5)
    m = m.eval().float()
    write_safetensors(str(tmp_path / "model.safetensors"), dict(m.state_dict()))
    d = m.config.to_dict()
    d["architectures"] = ["LlamaForCausalLM"]
    (tmp_path / "config.json").write_text(json.dumps(d))
    ours_cfg, tensors = load_reference_tensors_hf(str(tmp_path))
    assert dict(ours_cfg.rope_scaling)["type"] == params["rope_type"]
    ref = ReferenceModel(ours_cfg, tensors)
    ids = torch.tensor([3, 17, 200, 45, 9, 311, 7, 100, 250, 11])
    with torch.no_grad():
        want = m(ids[None]).logits[0]
    got = ref.forward(ids)
    assert torch.allclose(got, want, atol=2e-4, rtol=1e-4), (got - want).abs().max()
