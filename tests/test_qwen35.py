"""Qwen3.5 hybrid (Gated DeltaNet linear layers + gated full attention with partial rotary) on the
fp32 reference model, loaded from a Hugging Face checkpoint, against the transformers
implementation's logits (CPU); and token-at-a-time decoding through the recurrent state against
one full forward."""
import json

import pytest
import torch

transformers = pytest.importorskip("transformers")
if not hasattr(transformers, "Qwen3_5ForCausalLM"):
    pytest.skip("transformers has no Qwen3.5", allow_module_level=True)

from fak_b200.models.hf import load_reference_tensors_hf, write_safetensors  # noqa: E402
from fak_b200.models.reference import ReferenceModel  # noqa: E402

IDS = torch.tensor([3, 17, 200, 45, 9, 311, 7, 99, 12, 400, 5])


@pytest.fixture(scope="module")
def pair(tmp_path_factory):
    c = transformers.Qwen3_5TextConfig(vocab_size=512, hidden_size=128, intermediate_size=256, num_hidden_layers=3,
                                       num_attention_heads=4, num_key_value_heads=2, head_dim=32,
                                       linear_num_key_heads=2, linear_num_value_heads=4, linear_key_head_dim=16,
                                       linear_value_head_dim=24,
                                       layer_types=["linear_attention", "full_attention", "linear_attention"],
                                       max_position_embeddings=512)
    m = transformers.Qwen3_5ForCausalLM(c)
    m.config._attn_implementation = "eager"
    torch.manual_seed(0)
    for n, p in m.named_parameters():
        if n.endswith("A_log"):
            torch.nn.init.uniform_(p, -1.0, 1.0)
        else:
            torch.nn.init.normal_(p, std=0.08 if p.dim() > 1 else 0.3)
    m = m.eval().float()
    d = tmp_path_factory.mktemp("qwen35")
    write_safetensors(str(d / "model.safetensors"), dict(m.state_dict()))
    cfg = m.config.to_dict()
    cfg["architectures"] = [type(m).__name__]
    (d / "config.json").write_text(json.dumps(cfg))
    rcfg, tensors = load_reference_tensors_hf(str(d))
    return m, ReferenceModel(rcfg, tensors)


def test_qwen35_matches_transformers(pair):
    m, ref = pair
    cfg = ref.cfg
    assert cfg.arch == "qwen35" and cfg.linear_layers == (0, 2) and cfg.attn_out_gate and cfg.rope_dim == 8
    with torch.no_grad():
        want = m(IDS[None]).logits[0]
    got = ref.forward(IDS)
    assert torch.allclose(got, want, atol=3e-4, rtol=1e-4), (got - want).abs().max()


def test_qwen35_incremental_state_matches_full_forward(pair):
    """Prefill 6 tokens, then one token at a time: the conv tail and delta-rule state carried in
    the per-layer cache reproduce the logits of one forward over the whole sequence."""
    _, ref = pair
    full = ref.forward(IDS)
    kv: list = []
    out = [ref.forward(IDS[:6], 0, kv)]
    for t in range(6, len(IDS)):
        out.append(ref.forward(IDS[t:t + 1], t, kv))
    assert torch.allclose(torch.cat(out), full, atol=1e-4, rtol=1e-4)
