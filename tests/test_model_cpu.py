"""Reference forward, tokenizer, configs (CPU)."""
import numpy as np
import pytest
import torch

from fak_b200.config import EngineConfig, preset
from fak_b200.gguf.synth import write_synthetic_gguf
from fak_b200.models.loader import llama_rope_unpermute_rows
from fak_b200.gguf.synth import llama_rope_permute_rows
from fak_b200.models.reference import ReferenceModel, moe_route
from fak_b200.tokenizer import IncrementalDecoder, Tokenizer


@pytest.fixture(scope="module", params=["tiny-llama", "tiny-qwen2", "tiny-qwen3moe"])
def ref(request, tmp_path_factory):
    p = str(tmp_path_factory.mktemp("m") / f"{request.param}.gguf")
    write_synthetic_gguf(p, preset(request.param), "f32", seed=3)
    return ReferenceModel.from_gguf(p)


def test_incremental_equals_full(ref):
    ids = torch.arange(3, 40)
    full = ref.forward(ids)
    kv = []
    a = ref.forward(ids[:20], 0, kv)
    b = ref.forward(ids[20:], 20, kv)
    assert torch.allclose(full, torch.cat([a, b]), atol=1e-4)


def test_rope_permutation_roundtrip():
    rows = np.arange(4 * 64 * 3).reshape(4 * 64, 3)
    p = llama_rope_permute_rows(rows, 4, 64)
    assert not (p == rows).all()
    assert (llama_rope_unpermute_rows(p, 4, 64) == rows).all()


def test_moe_router_semantics():
    logits = torch.tensor([[1.0, 3.0, 2.0, 0.0]])
    w, idx = moe_route(logits, 2, True)
    assert idx.tolist() == [[1, 2]]
    assert torch.allclose(w.sum(-1), torch.tensor([1.0]))
    w2, _ = moe_route(logits, 2, False)
    assert w2.sum() < 1.0


def test_tokenizer_roundtrip_and_specials(tmp_path):
    p = str(tmp_path / "t.gguf")
    write_synthetic_gguf(p, preset("tiny-qwen2"), "q8_0")
    from fak_b200.gguf import open_gguf
    tok = Tokenizer.from_gguf_metadata(open_gguf(p).metadata)
    text = "<|im_start|>user\nHello wörld, the cat sat! 12 <|im_end|>"
    ids = tok.encode(text)
    assert tok.decode(ids) == text
    assert tok.token_to_id["<|im_start|>"] in ids
    dec = IncrementalDecoder(tok, skip_special=False)
    s = "".join(dec.push(i) for i in ids) + dec.flush()
    assert s == text


def test_engine_config_env(monkeypatch):
    monkeypatch.setenv("FAK_PAGED_KV_BLOCK_TOKENS", "16")
    monkeypatch.setenv("FAK_CUDA_GRAPH", "0")
    monkeypatch.setenv("FAK_NATIVE_MAX_RUNNING", "12")
    e = EngineConfig.from_env()
    assert e.cuda_graph is False and e.max_batch == 12 and e.page_size == 16
    e2 = EngineConfig.from_env(max_batch=3)
    assert e2.max_batch == 3


def test_param_counts():
    assert 7.0e9 < preset("qwen2.5-7b").param_count() < 7.8e9
    assert 1.2e8 < preset("smollm2-135m").param_count() < 1.5e8
    assert 2.9e10 < preset("qwen3-30b-a3b").param_count() < 3.2e10


def test_dsa_reference_definitions():
    """Sparse-attention definitions: top-k order (score, then position) and attention over the full
    set equal to dense softmax attention."""
    import math
    from fak_b200.models.dsa import index_scores_ref, sparse_attend_ref, topk_ref
    g = torch.Generator().manual_seed(0)
    iq, ik, w = torch.randn(4, 8, generator=g), torch.randn(20, 8, generator=g), torch.rand(4, generator=g)
    ik[5] = ik[2]
    s = index_scores_ref(iq, ik, w, 15, 0.5)
    assert torch.isinf(s[16:]).all()
    sel = topk_ref(s, 15, 6)
    assert len(sel) == 6 and sorted(s[sel].tolist(), reverse=True) == s[sel].tolist()
    if 2 in sel or 5 in sel:
        assert (2 in sel) and (sel.index(2) < sel.index(5) if 5 in sel else True)
    q, kc, vc = torch.randn(3, 6, generator=g), torch.randn(20, 3, 6, generator=g), torch.randn(20, 3, 4, generator=g)
    full = sparse_attend_ref(q, kc, vc, list(range(20)), 1 / math.sqrt(6))
    dense = torch.softmax(torch.einsum("hd,nhd->hn", q, kc) / math.sqrt(6), -1)
    assert torch.allclose(full, torch.einsum("hn,nhv->hv", dense, vc), atol=1e-6)
