"""Gemma-4 dense text decoder on the fp32 reference path (per-layer head geometry, k-as-v global
layers, q/k/v norms, scale 1, proportional RoPE, sandwich norms, layer scalars) against the
transformers implementation's logits (CPU)."""
import json

import pytest
import torch

transformers = pytest.importorskip("transformers")
if not hasattr(transformers, "Gemma4ForCausalLM"):
    pytest.skip("transformers has no Gemma-4", allow_module_level=True)

from fak_b200.models.gemma4 import Gemma4Reference  # noqa: E402
from fak_b200.models.hf import write_safetensors  # noqa: E402


@pytest.mark.parametrize("k_eq_v,softcap", [(True, 30.0), (False, None)])
def test_gemma4_matches_transformers(tmp_path, k_eq_v, softcap):
    c = transformers.Gemma4TextConfig(
        vocab_size=512, hidden_size=128, intermediate_size=256, num_hidden_layers=3, num_attention_heads=4,
        num_key_value_heads=2, head_dim=32, global_head_dim=64, num_global_key_value_heads=1 if k_eq_v else None,
        attention_k_eq_v=k_eq_v, sliding_window=4, layer_types=["sliding_attention", "full_attention", "sliding_attention"],
        hidden_size_per_layer_input=0, vocab_size_per_layer_input=512, final_logit_softcapping=softcap,
        max_position_embeddings=256,
        rope_parameters={"sliding_attention": {"rope_type": "default", "rope_theta": 10000.0},
                         "full_attention": {"rope_type": "proportional", "partial_rotary_factor": 0.25,
                                            "rope_theta": 1000000.0}})
    m = transformers.Gemma4ForCausalLM(c)
    m.config._attn_implementation = "eager"
    torch.manual_seed(0)
    for n, p in m.named_parameters():
        torch.nn.init.normal_(p, std=0.08 if p.dim() > 1 else 0.3)
        if p.dim() == 1:
            p.data += 1.0
    for n, b in m.named_buffers():
        if n.endswith("layer_scalar"):
            b.fill_(0.7)
    m = m.eval().float()
    write_safetensors(str(tmp_path / "model.safetensors"), dict(m.state_dict()))
    cfg = m.config.to_dict()
    cfg["architectures"] = [type(m).__name__]
    (tmp_path / "config.json").write_text(json.dumps(cfg))
    ref = Gemma4Reference.from_hf(str(tmp_path))
    ids = torch.tensor([3, 17, 200, 45, 9, 311, 7, 99, 12, 400, 5])
    with torch.no_grad():
        want = m(ids[None]).logits[0]
    got = ref.forward(ids)
    assert torch.allclose(got, want, atol=3e-4, rtol=1e-4), (got - want).abs().max()


def test_cacheless_adapter_serves_a_whole_sequence_model():
    """The reference backend drives whole-sequence models through CachelessModel: greedy tokens
    equal the argmax chain of full forwards over the growing sequence."""
    from fak_b200.engine.sampling import SamplingParams
    from fak_b200.serve.backend import CachelessModel, ReferenceBackend

    class Whole:
        V = 37

        def forward(self, ids):
            ids = torch.as_tensor(ids)
            cs = torch.cumsum(ids * torch.arange(1, ids.numel() + 1), 0)
            return torch.nn.functional.one_hot((cs * 7 + 3) % self.V, self.V).float()

    m = Whole()
    be = ReferenceBackend(CachelessModel(m), tokenizer=None)
    got = list(be.generate([5, 11, 2], 6, SamplingParams()))
    seq, want = [5, 11, 2], []
    for _ in range(6):
        t = int(m.forward(seq)[-1].argmax())
        want.append(t)
        seq.append(t)
    assert got == want
    with pytest.raises(ValueError):
        CachelessModel(m).forward(torch.tensor([1]), 3, [])
