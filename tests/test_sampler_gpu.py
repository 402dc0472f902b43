"""The device sampler (``csrc/kernels/sampler.cu``) against an fp64 reference of the same semantics, and
the engine's sampled decode steps (GPU only)."""
import math

import numpy as np
import pytest
import torch

from fak_b200.engine.sampling import SamplingParams, count_rows, pack_params

pytestmark = pytest.mark.gpu


def _run(logits, sps, steps, seeds, generated=None, softcap=0.0):
    from fak_b200.ops import kernels as K
    n, V = logits.shape
    P, tok, val = pack_params(sps, steps, seeds, max_bias=None)
    p = torch.from_numpy(P).cuda()
    bt = torch.from_numpy(tok if len(tok) else np.full(1, -1, np.int32)).cuda()
    bv = torch.from_numpy(val if len(val) else np.zeros(1, np.float32)).cuda()
    counts = count_rows(generated, V, "cuda") if generated is not None else None
    out = torch.empty(n, dtype=torch.int32, device="cuda")
    x = logits.clone()
    K.sample_rows(x, V, p, bt, bv, counts, out, n, softcap)
    torch.cuda.synchronize()
    return out.cpu().numpy(), p.cpu().numpy(), x


def _reference_probs(logits: np.ndarray, sp: SamplingParams, counts=None) -> np.ndarray:
    """fp64 distribution of the documented semantics (ties at the top-k / top-p boundary kept)."""
    x = logits.astype(np.float64).copy()
    if counts is not None:
        x -= sp.frequency_penalty * counts + sp.presence_penalty * (counts > 0)
    for t, b in (sp.logit_bias or {}).items():
        x[t] += max(-100.0, min(100.0, b))
    x /= sp.temperature
    p = np.exp(x - x.max())
    keep = np.ones_like(p, bool)
    if 0 < sp.top_k < len(p):
        kth = np.sort(x)[::-1][sp.top_k - 1]
        keep &= x >= kth
    if 0 < sp.top_p < 1:
        order = np.argsort(-p, kind="stable")
        mass = np.where(keep, p, 0.0)
        cum = np.cumsum(mass[order])
        target = sp.top_p * mass.sum()
        cut = int(np.searchsorted(cum, target))          # first rank where cum >= target
        thr = p[order[min(cut, len(p) - 1)]]
        keep &= p >= thr
    q = np.where(keep, p, 0.0)
    return q / q.sum()


def test_greedy_rows_are_first_index_argmax_after_bias_and_penalties():
    g = torch.Generator(device="cuda").manual_seed(0)
    V = 50000
    logits = torch.randn(6, V, device="cuda", generator=g)
    logits[1, 17] = logits[1, 99] = logits[1].max() + 1.0            # a tie: first index wins
    sps = [SamplingParams(), SamplingParams(), SamplingParams(logit_bias={123: 1000.0}),
           SamplingParams(frequency_penalty=5.0), SamplingParams(presence_penalty=50.0),
           SamplingParams(logit_bias={5: -1000.0})]
    gen = [[], [], [], [int(logits[3].argmax())] * 2, [int(logits[4].argmax())], []]
    got, P, _ = _run(logits, sps, [0] * 6, [1] * 6, gen)
    ref = logits.clone()
    ref[2, 123] += 100.0
    ref[3, int(logits[3].argmax())] -= 10.0
    ref[4, int(logits[4].argmax())] -= 50.0
    ref[5, 5] -= 100.0
    assert got.tolist() == ref.argmax(1).tolist()
    assert got[1] == 17
    assert (P[:, 9] == 1).all(), "the draw counter advances"


@pytest.mark.parametrize("sp", [SamplingParams(temperature=0.8),
                                SamplingParams(temperature=0.7, top_k=20),
                                SamplingParams(temperature=1.3, top_p=0.8),
                                SamplingParams(temperature=0.9, top_k=40, top_p=0.6,
                                               logit_bias={3: 2.0, 11: -3.0})])
def test_draws_follow_the_reference_distribution(sp):
    V, N = 512, 40000
    g = torch.Generator(device="cuda").manual_seed(3)
    row = torch.randn(V, device="cuda", generator=g) * 2.0
    logits = row.expand(N, V).contiguous()
    got, _, _ = _run(logits, [sp] * N, list(range(N)), [0xC0FFEE] * N)
    want = _reference_probs(row.cpu().numpy(), sp)
    emp = np.bincount(got, minlength=V) / N
    assert set(np.nonzero(emp)[0]) <= set(np.nonzero(want)[0]), "a token outside the kept set was drawn"
    tv = 0.5 * np.abs(emp - want).sum()
    k = int((want > 0).sum())
    # twice the multinomial bound E[TV] <= sqrt(2 k / (pi N)) / 2, plus a little slack
    assert tv < math.sqrt(2 * k / (math.pi * N)) + 0.01, (tv, k)


def test_draw_is_keyed_by_seed_and_step():
    V = 4096
    g = torch.Generator(device="cuda").manual_seed(5)
    row = torch.randn(V, device="cuda", generator=g)
    logits = row.expand(64, V).contiguous()
    sp = SamplingParams(temperature=1.0)
    a, _, _ = _run(logits, [sp] * 64, [7] * 64, [42] * 64)
    assert len(set(a.tolist())) == 1, "same (seed, step) -> same token in every row"
    b, _, _ = _run(logits, [sp] * 64, list(range(64)), [42] * 64)
    c, _, _ = _run(logits, [sp] * 64, list(range(64)), [43] * 64)
    assert len(set(b.tolist())) > 10 and b.tolist() != c.tolist()
    d, _, _ = _run(logits, [sp] * 64, list(range(64)), [42] * 64)
    assert b.tolist() == d.tolist(), "deterministic"


def test_soft_cap_changes_the_distribution_like_the_host_cap():
    V, N = 256, 30000
    g = torch.Generator(device="cuda").manual_seed(9)
    row = torch.randn(V, device="cuda", generator=g) * 8.0
    logits = row.expand(N, V).contiguous()
    sp = SamplingParams(temperature=1.0)
    got, _, _ = _run(logits, [sp] * N, list(range(N)), [1] * N, softcap=5.0)
    capped = 5.0 * np.tanh(row.cpu().numpy().astype(np.float64) / 5.0)
    want = _reference_probs(capped, sp)
    emp = np.bincount(got, minlength=V) / N
    k = int((want > 0).sum())
    assert 0.5 * np.abs(emp - want).sum() < math.sqrt(2 * k / (math.pi * N)) + 0.01


def test_engine_sampled_async_equals_sync_and_mixed_batches(tmp_path):
    """Sampled lanes through the device-resident loop draw exactly what the synchronous loop draws
    (the draw depends on the request's seed and step only), and greedy lanes in a sampled batch
    decode as they do alone."""
    from fak_b200.config import EngineConfig, preset
    from fak_b200.engine import Engine
    from fak_b200.gguf.synth import write_synthetic_gguf
    path = str(tmp_path / "m.gguf")
    write_synthetic_gguf(path, preset("tiny-qwen2"), "q4_k_m", seed=5, std=0.05)

    def run(async_decode):
        ecfg = EngineConfig(max_batch=8, kv_pages=512, cuda_graph=True, graph_batch_buckets=(1, 2, 4, 8),
                            async_decode=async_decode)
        eng = Engine.from_gguf(path, ecfg, "cuda", max_context=1024)
        eng.warmup_graphs()
        rng = np.random.default_rng(11)
        V = eng.cfg.vocab_size
        sps = [SamplingParams(temperature=0.8, top_p=0.9, seed=1), SamplingParams(),
               SamplingParams(temperature=1.1, top_k=30, frequency_penalty=0.7, presence_penalty=0.3, seed=7),
               SamplingParams(temperature=0.6, logit_bias={5: 4.0}, seed=3)]
        reqs = [eng.add_request(rng.integers(0, V, n).tolist(), 20, sp) for n, sp in zip((30, 9, 44, 17), sps)]
        eng.run_until_done(reqs)
        return [r.full_output for r in reqs], eng

    want, _ = run(False)
    got, eng = run(True)
    assert got == want
    rng = np.random.default_rng(11)
    rng.integers(0, eng.cfg.vocab_size, 30)
    alone = eng.generate([rng.integers(0, eng.cfg.vocab_size, 9).tolist()], 20)[0]
    assert got[1] == alone, "a greedy lane decodes the same inside a sampled batch"
