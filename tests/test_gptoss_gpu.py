"""gpt-oss on the device engine: attention sinks, biased q/k/v/o, the biased top-k-then-softmax
router, biased experts with the clamped gate, alternating sliding windows and YaRN, from a Hugging
Face checkpoint (float, quantized to Q8_0 on load) against the fp32 reference model."""
import json

import numpy as np
import pytest
import torch

transformers = pytest.importorskip("transformers")

pytestmark = pytest.mark.gpu


def _checkpoint(tmp_path):
    from fak_b200.models.hf import write_safetensors
    c = transformers.GptOssConfig(vocab_size=512, hidden_size=256, intermediate_size=256, num_hidden_layers=2,
                                  num_attention_heads=4, num_key_value_heads=2, head_dim=64, num_local_experts=4,
                                  num_experts_per_tok=2, sliding_window=16, max_position_embeddings=1024,
                                  rope_parameters={"rope_type": "yarn", "factor": 8.0, "beta_fast": 32.0,
                                                   "beta_slow": 1.0, "truncate": False, "rope_theta": 150000.0,
                                                   "original_max_position_embeddings": 128})
    m = transformers.GptOssForCausalLM(c)
    torch.manual_seed(3)
    for _, p in m.named_parameters():
        torch.nn.init.normal_(p, std=0.05 if p.dim() > 1 else 0.5)
    write_safetensors(str(tmp_path / "model.safetensors"), dict(m.state_dict()))
    cfg = m.config.to_dict()
    cfg["architectures"] = [type(m).__name__]
    (tmp_path / "config.json").write_text(json.dumps(cfg))
    return str(tmp_path)


def test_gptoss_engine_matches_reference(tmp_path):
    from fak_b200.config import EngineConfig
    from fak_b200.engine import Engine
    from fak_b200.models.hf import load_reference_tensors_hf
    from fak_b200.models.reference import ReferenceModel
    d = _checkpoint(tmp_path)
    cfg, tensors = load_reference_tensors_hf(d)
    assert cfg.attn_sinks and cfg.moe_bias and cfg.router == "topk_softmax" and cfg.device_gap() is None
    ref = ReferenceModel(cfg, tensors, "cuda")
    prompt = np.random.default_rng(5).integers(0, cfg.vocab_size, 40).tolist()
    eng = Engine.from_hf(d, EngineConfig(max_batch=4, kv_pages=256, cuda_graph=True, graph_batch_buckets=(1, 2)),
                         "cuda", max_context=512)
    eng.warmup_graphs()
    from fak_b200.benchmarks.tpcheck import forced_logits
    want_ids = ref.generate_greedy(prompt, 12)
    got_logits = forced_logits(eng, prompt, want_ids[:-1])
    with torch.no_grad():
        ref_logits = ref.forward(torch.tensor(prompt + want_ids[:-1]))[len(prompt) - 1:].float().cpu()
    V = cfg.vocab_size
    got_logits, ref_logits = got_logits[:, :V], ref_logits[:, :V]
    cos = torch.nn.functional.cosine_similarity(got_logits, ref_logits, dim=1)
    assert float(cos.min()) > 0.99, cos
    agree = (got_logits.argmax(1) == ref_logits.argmax(1)).float().mean().item()
    assert agree >= 0.75, agree
    out = eng.generate([prompt], max_new_tokens=12)[0]
    eng.shutdown()
    k = 0
    while k < len(out) and out[k] == want_ids[k]:
        k += 1
    if k < len(out):
        # up to the first difference both runs saw the same tokens, so row k of the teacher-forced
        # logits is the engine's own step k: the difference must be a near-tie of the fp32 model
        # (its gap between the two tokens within twice the measured logit error on them)
        a, b = want_ids[k], out[k]
        gap = float(ref_logits[k, a] - ref_logits[k, b])
        err = float((got_logits[k, a] - ref_logits[k, a]).abs() + (got_logits[k, b] - ref_logits[k, b]).abs())
        assert gap <= max(0.05, 2.0 * err), (k, gap, err, out, want_ids)
