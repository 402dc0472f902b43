"""Governed text + image prompts on the reference model: fail-closed admission (quarantine by
default, limits, content types, shapes) and the splice of image rows into the sequence."""
import pytest
import torch

from fak_b200.config import preset
from fak_b200.models import multimodal as mm
from fak_b200.models.reference import ReferenceModel


@pytest.fixture(scope="module")
def model():
    cfg = preset("tiny-llama")
    g = torch.Generator().manual_seed(0)
    shapes = {"token_embd.weight": (cfg.vocab_size, cfg.d_model), "output_norm.weight": (cfg.d_model,)}
    for i in range(cfg.n_layers):
        p = f"blk.{i}."
        shapes.update({p + "attn_norm.weight": (cfg.d_model,), p + "ffn_norm.weight": (cfg.d_model,),
                       p + "attn_q.weight": (cfg.q_dim, cfg.d_model), p + "attn_k.weight": (cfg.kv_dim, cfg.d_model),
                       p + "attn_v.weight": (cfg.kv_dim, cfg.d_model), p + "attn_output.weight": (cfg.d_model, cfg.q_dim),
                       p + "ffn_gate.weight": (cfg.ffn_dim, cfg.d_model), p + "ffn_up.weight": (cfg.ffn_dim, cfg.d_model),
                       p + "ffn_down.weight": (cfg.d_model, cfg.ffn_dim)})
    t = {k: (1.0 + 0.1 * torch.randn(s, generator=g)) if len(s) == 1 else 0.05 * torch.randn(s, generator=g)
         for k, s in shapes.items()}
    return ReferenceModel(cfg, t)


def _img(model, n=3, media="image/png", w=32, h=32, data=b"\x89PNG....", seed=1):
    g = torch.Generator().manual_seed(seed)
    return mm.VisionEmbedding(mm.Image(media, w, h, data), torch.randn(n, model.cfg.d_model, generator=g))


def test_text_only_runs_under_the_default_policy_and_matches_forward(model):
    ids = [5, 9, 100, 7]
    logits, v = mm.forward_multimodal(model, [mm.Part(token_ids=ids)])
    assert v.decision == "allow" and v.images == 0
    assert torch.allclose(logits, model.forward(torch.tensor(ids)), atol=1e-5)


def test_images_are_quarantined_until_opt_in(model):
    parts = [mm.Part(token_ids=[1, 2]), mm.Part(image=_img(model)), mm.Part(token_ids=[3])]
    with pytest.raises(mm.MultimodalQuarantined) as e:
        mm.prepare_rows(model, parts)
    v = e.value.verdict
    assert v.decision == "quarantine" and v.images == 1 and v.embedding_tokens == 3
    qid = mm.quarantine_id(parts)
    assert qid.startswith("vision-sha256:") and qid == v.quarantine_id
    assert qid != mm.quarantine_id([mm.Part(image=_img(model, seed=2))])
    rows, v = mm.prepare_rows(model, parts, mm.Policy(mode="quarantine"))
    assert v.decision == "allow" and v.images == 1 and v.embedding_tokens == 3 and rows.shape == (6, model.cfg.d_model)
    assert torch.equal(rows[2:5], parts[1].image.vectors)             # image rows enter unchanged
    assert torch.allclose(rows[:2], model.embed(torch.tensor([1, 2])))
    logits, _ = mm.forward_multimodal(model, parts, mm.Policy(mode="quarantine"))
    assert logits.shape == (6, model.cfg.vocab_size) and torch.isfinite(logits).all()


@pytest.mark.parametrize("make,reason", [
    (lambda m: [mm.Part(image=_img(m, media="image/svg+xml"))], "allow-list"),
    (lambda m: [mm.Part(image=_img(m, media="text/plain"))], "image/*"),
    (lambda m: [mm.Part(image=_img(m, w=0))], "dimensions"),
    (lambda m: [mm.Part(image=_img(m, w=5000, h=5000))], "pixel"),
    (lambda m: [mm.Part(image=_img(m, data=b"x" * (11 << 20)))], "bytes"),
    (lambda m: [mm.Part(image=_img(m, n=0))], "empty"),
    (lambda m: [mm.Part(image=_img(m, n=1025))], "token count"),
    (lambda m: [mm.Part(image=_img(m))] * 5, "too many"),
    (lambda m: [mm.Part(token_ids=[1], image=_img(m))], "exactly one"),
    (lambda m: [mm.Part(token_ids=[10 ** 6])], "vocab"),
    (lambda m: [], "empty prompt"),
])
def test_violations_deny_the_whole_prompt(model, make, reason):
    with pytest.raises(mm.MultimodalDenied, match=reason) as e:
        mm.prepare_rows(model, make(model), mm.Policy(mode="quarantine"))
    assert e.value.verdict.decision == "deny"


def test_wrong_width_and_policy_checks(model):
    bad = mm.VisionEmbedding(mm.Image("image/png", 4, 4), torch.zeros(2, model.cfg.d_model + 1))
    with pytest.raises(mm.MultimodalDenied, match="width"):
        mm.prepare_rows(model, [mm.Part(image=bad)], mm.Policy(mode="quarantine"))
    with pytest.raises(mm.MultimodalDenied, match="mode"):
        mm.prepare_rows(model, [mm.Part(token_ids=[1])], mm.Policy(mode="open"))
    with pytest.raises(mm.MultimodalDenied, match="media type"):
        mm.prepare_rows(model, [mm.Part(token_ids=[1])], mm.Policy(allowed_content_types=("text/html",)))
    # parameters and case are ignored on the content-type axis; wildcards widen it
    ok = _img(model, media="Image/PNG; charset=binary")
    mm.prepare_rows(model, [mm.Part(image=ok)], mm.Policy(mode="quarantine"))
    tiff = _img(model, media="image/tiff")
    mm.prepare_rows(model, [mm.Part(image=tiff)], mm.Policy(mode="quarantine", allowed_content_types=("image/*",)))
