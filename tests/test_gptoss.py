"""gpt-oss blocks on the fp32 reference model: attention sinks, biased top-k-then-softmax router,
clamped OAI gate, alternating windows, YaRN; loaded from a Hugging Face checkpoint in float form
and in MXFP4 form, against the transformers implementation's logits (CPU)."""
import json

import numpy as np
import pytest
import torch

transformers = pytest.importorskip("transformers")

from fak_b200.models import mxfp4  # noqa: E402
from fak_b200.models.hf import load_reference_tensors_hf, write_safetensors  # noqa: E402
from fak_b200.models.reference import ReferenceModel, attention  # noqa: E402


def _model(seed=0):
    c = transformers.GptOssConfig(vocab_size=512, hidden_size=128, intermediate_size=64, num_hidden_layers=2,
                                  num_attention_heads=4, num_key_value_heads=2, head_dim=32, num_local_experts=4,
                                  num_experts_per_tok=2, sliding_window=6, max_position_embeddings=512,
                                  rope_parameters={"rope_type": "yarn", "factor": 8.0, "beta_fast": 32.0,
                                                   "beta_slow": 1.0, "truncate": False, "rope_theta": 150000.0,
                                                   "original_max_position_embeddings": 64})
    m = transformers.GptOssForCausalLM(c)
    m.config._attn_implementation = "eager"
    torch.manual_seed(seed)
    for n, p in m.named_parameters():
        torch.nn.init.normal_(p, std=0.08 if p.dim() > 1 else 0.5)
    return m.eval().float()


def _save(m, tmp_path, tensors):
    write_safetensors(str(tmp_path / "model.safetensors"), tensors)
    cfg = m.config.to_dict()
    cfg["architectures"] = [type(m).__name__]
    (tmp_path / "config.json").write_text(json.dumps(cfg))
    return str(tmp_path)


IDS = torch.tensor([3, 17, 200, 45, 9, 311, 7, 99, 12, 400, 5])


def test_gptoss_float_checkpoint_matches_transformers(tmp_path):
    m = _model()
    d = _save(m, tmp_path, dict(m.state_dict()))
    cfg, tensors = load_reference_tensors_hf(d)
    assert cfg.arch == "gptoss" and cfg.attn_sinks and cfg.router == "topk_softmax" and cfg.moe_bias
    assert [cfg.layer_window(i) for i in range(2)] == [6, 0]
    ref = ReferenceModel(cfg, tensors)
    with torch.no_grad():
        want = m(IDS[None]).logits[0]
    got = ref.forward(IDS)
    assert torch.allclose(got, want, atol=3e-4, rtol=1e-4), (got - want).abs().max()


def test_gptoss_mxfp4_checkpoint_matches_transformers(tmp_path):
    """Experts stored as MXFP4 blocks + scales (out-major); transformers runs the same dequantized
    values in its float layout."""
    m = _model(1)
    sd = dict(m.state_dict())
    out = {}
    for k, v in sd.items():
        if k.endswith("experts.gate_up_proj") or k.endswith("experts.down_proj"):
            w = v.transpose(1, 2).contiguous().numpy()            # [E, out, in]
            blocks, scales = mxfp4.quantize(w)
            out[k + "_blocks"] = torch.from_numpy(blocks)
            out[k + "_scales"] = torch.from_numpy(scales)
            deq = torch.from_numpy(mxfp4.dequantize(blocks, scales)).transpose(1, 2).contiguous()
            with torch.no_grad():   # the oracle runs on exactly the values the checkpoint holds
                dict(m.named_parameters())[k].copy_(deq)
        else:
            out[k] = v
    d = _save(m, tmp_path, out)
    cfg, tensors = load_reference_tensors_hf(d)
    ref = ReferenceModel(cfg, tensors)
    with torch.no_grad():
        want = m(IDS[None]).logits[0]
    got = ref.forward(IDS)
    assert torch.allclose(got, want, atol=3e-4, rtol=1e-4), (got - want).abs().max()


def test_mxfp4_roundtrip_and_layout():
    rng = np.random.default_rng(0)
    w = rng.standard_normal((3, 5, 64)).astype(np.float32)
    blocks, scales = mxfp4.quantize(w)
    assert blocks.shape == (3, 5, 2, 16) and scales.shape == (3, 5, 2) and blocks.dtype == np.uint8
    back = mxfp4.dequantize(blocks, scales)
    # neighbouring E2M1 magnitudes are at most 2 apart (4 and 6), so rounding is off by at most one
    # block scale, and by at most a third of the value above magnitude 1.5
    scale = np.ldexp(1.0, scales.astype(np.int32) - 127).repeat(32, axis=-1)
    assert np.all(np.abs(back - w) <= scale + 1e-6)
    big = np.abs(w) >= 1.5 * scale
    assert np.all(np.abs(back - w)[big] <= np.abs(w)[big] / 3 + 1e-6)
    # a hand-built block: low nibble first; codes 1 (0.5) and 0xF (-6); scale 2^1
    b = np.zeros((1, 16), np.uint8)
    b[0, 0] = 0xF1
    v = mxfp4.dequantize(b, np.array([128], np.uint8))
    assert v[0] == 1.0 and v[1] == -12.0 and np.all(v[2:] == 0)


def test_sink_softmax_matches_the_explicit_form():
    torch.manual_seed(0)
    q, K, V = torch.randn(3, 4, 16), torch.randn(7, 2, 16), torch.randn(7, 2, 16)
    sinks = torch.tensor([0.5, -1.0, 2.0, 0.0])
    got = attention(q, K, V, 4, sinks=sinks)
    Kx, Vx = K.repeat_interleave(2, 1), V.repeat_interleave(2, 1)
    for h in range(4):
        for t in range(3):
            s = (Kx[: 5 + t, h] @ q[t, h]) / 4.0
            e = torch.exp(s - s.max())
            den = e.sum() + torch.exp(sinks[h] - s.max())
            assert torch.allclose(got[t, h], (e[:, None] * Vx[: 5 + t, h]).sum(0) / den, atol=1e-5)


@pytest.mark.parametrize("name", ["tiny-gptoss", "gpt-oss-20b"])
def test_device_engine_takes_gptoss_and_refuses_other_gate_constants(name):
    """The device kernels carry gpt-oss's gate constants (alpha 1.702, limit 7): the family runs on
    the device engine, a model with other constants is refused before any weight is loaded."""
    from fak_b200.config import preset
    from fak_b200.engine import Engine
    cfg = preset(name)
    assert cfg.device_gap() is None
    odd = cfg.replace(swiglu_alpha=1.5)
    assert "1.702" in odd.device_gap()
    with pytest.raises(NotImplementedError, match="reference model"):
        Engine.synthetic(odd, device="cpu")
    assert preset("qwen2.5-7b").device_gap() is None
