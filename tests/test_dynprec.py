"""Dynamic precision on the reference path: Q8_0 steps accepted only when confident, rejected
steps rolled back and recomputed in fp32, against fixed fp32 / fixed Q8_0 runs."""
import torch

from fak_b200.config import preset
from fak_b200.models.dynprec import DynamicPrecisionSession, q8_0_round
from fak_b200.models.reference import ReferenceModel


def _model():
    cfg = preset("tiny-llama")
    g = torch.Generator().manual_seed(1)
    shapes = {"token_embd.weight": (cfg.vocab_size, cfg.d_model), "output_norm.weight": (cfg.d_model,)}
    for i in range(cfg.n_layers):
        p = f"blk.{i}."
        shapes.update({p + "attn_norm.weight": (cfg.d_model,), p + "ffn_norm.weight": (cfg.d_model,),
                       p + "attn_q.weight": (cfg.q_dim, cfg.d_model), p + "attn_k.weight": (cfg.kv_dim, cfg.d_model),
                       p + "attn_v.weight": (cfg.kv_dim, cfg.d_model), p + "attn_output.weight": (cfg.d_model, cfg.q_dim),
                       p + "ffn_gate.weight": (cfg.ffn_dim, cfg.d_model), p + "ffn_up.weight": (cfg.ffn_dim, cfg.d_model),
                       p + "ffn_down.weight": (cfg.d_model, cfg.ffn_dim)})
    t = {k: (1.0 + 0.1 * torch.randn(s, generator=g)) if len(s) == 1 else 0.08 * torch.randn(s, generator=g)
         for k, s in shapes.items()}
    return ReferenceModel(cfg, t)


PROMPT = [5, 9, 100, 7, 33, 250]


def test_accept_all_equals_a_fixed_q8_run():
    m = _model()
    s = DynamicPrecisionSession(m)
    got = s.generate_greedy(PROMPT, 6)
    assert got == s.q8.generate_greedy(PROMPT, 6)
    assert s.stats.rejected == 0 and s.stats.q8_tokens == len(PROMPT) + 6 and s.stats.f32_tokens == 0


def test_reject_all_rolls_back_and_equals_fp32():
    m = _model()
    s = DynamicPrecisionSession(m, min_prob=1.01)          # never confident enough
    got = s.generate_greedy(PROMPT, 6)
    assert got == m.generate_greedy(PROMPT, 6)
    assert s.stats.accepted == 0 and s.stats.f32_tokens == len(PROMPT) + 6
    # the rolled-back cache holds fp32 keys only: the next logits match a pure fp32 forward
    nxt = s.run([got[-1]])
    ref = m.forward(torch.tensor(PROMPT + got + [got[-1]]))[-1]
    assert torch.allclose(nxt, ref, atol=1e-4)


def test_mixed_decisions_follow_the_margin_gate():
    m = _model()
    s = DynamicPrecisionSession(m, min_margin=1e9)
    s.run(PROMPT)
    assert s.stats.rejected == 1 and not s.accepts(s.stats.last_margin, s.stats.last_prob)
    s.min_margin = 0.0
    s.run([3])
    assert s.stats.accepted == 1 and s.stats.q8_tokens == 1 and s.pos == len(PROMPT) + 1


def test_q8_rounding_is_close_but_not_exact():
    w = torch.randn(8, 64)
    r = q8_0_round(w)
    assert not torch.equal(r, w) and float((r - w).abs().max()) < float(w.abs().max()) / 100
