"""GLM-MoE-DSA on the fp32 reference path: MLA with DSA-indexer key selection, sigmoid
group-limited MoE with shared experts, dense first layers -- against the transformers
implementation's logits (CPU), with the indexer's top-k small enough to drop keys."""
import json

import pytest
import torch

transformers = pytest.importorskip("transformers")
if not hasattr(transformers, "GlmMoeDsaForCausalLM"):
    pytest.skip("transformers has no GLM-MoE-DSA", allow_module_level=True)

from fak_b200.models.glm_dsa import GlmDsaReference  # noqa: E402
from fak_b200.models.hf import write_safetensors  # noqa: E402


@pytest.mark.parametrize("index_topk,q_lora", [(4, 48), (64, 48), (5, 64)])
def test_glm_dsa_matches_transformers(tmp_path, index_topk, q_lora):
    c = transformers.GlmMoeDsaConfig(vocab_size=512, hidden_size=128, intermediate_size=192, moe_intermediate_size=32,
                                     num_hidden_layers=3, num_attention_heads=4, num_key_value_heads=4,
                                     n_shared_experts=1, n_routed_experts=8, routed_scaling_factor=2.5,
                                     kv_lora_rank=32, q_lora_rank=q_lora, qk_rope_head_dim=16, v_head_dim=24,
                                     qk_nope_head_dim=24, n_group=2, topk_group=1, num_experts_per_tok=2,
                                     index_topk=index_topk, index_head_dim=32, index_n_heads=4,
                                     max_position_embeddings=256, mlp_layer_types=["dense", "sparse", "sparse"])
    m = transformers.GlmMoeDsaForCausalLM(c)
    m.config._attn_implementation = "eager"
    torch.manual_seed(0)
    for n, p in m.named_parameters():
        torch.nn.init.normal_(p, std=0.08 if p.dim() > 1 else 0.3)
    for n, b in m.named_buffers():
        if n.endswith("e_score_correction_bias"):
            b.copy_(0.1 * torch.randn_like(b))
    m = m.eval().float()
    sd = {k: v for k, v in m.state_dict().items()}
    write_safetensors(str(tmp_path / "model.safetensors"), sd)
    cfg = m.config.to_dict()
    cfg["architectures"] = [type(m).__name__]
    (tmp_path / "config.json").write_text(json.dumps(cfg))
    ref = GlmDsaReference.from_hf(str(tmp_path))
    ids = torch.tensor([3, 17, 200, 45, 9, 311, 7, 99, 12, 400, 5])
    with torch.no_grad():
        want = m(ids[None]).logits[0]
    got = ref.forward(ids)
    assert torch.allclose(got, want, atol=3e-4, rtol=1e-4), (got - want).abs().max()
