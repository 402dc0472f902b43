"""Capacity planner and roofline model (CPU)."""
import math

import pytest

from fak_b200 import capacity as C
from fak_b200.config import preset
from fak_b200.utils import roofline as R


def test_plan_weights_match_the_model_size():
    cfg = preset("qwen2.5-7b")
    p = C.plan(cfg, "q4_k_m", max_context=2048, batch=1)
    # ~7.6e9 params at ~0.6 B/weight (Q4_K_M) -> 4-5 GB of blocks
    assert 4.0e9 < p.weights < 5.5e9
    assert p.prefill_bf16 > 2 * p.tile_packed  # bf16 copies are ~3.3x the 4.5-bit blocks
    assert p.kv == p.kv_pages * 16 * C.kv_bytes_per_token(cfg)
    assert C.kv_bytes_per_token(cfg) == 28 * 2 * 4 * 128 * 2


def test_tp_and_ep_shrink_the_per_rank_plan():
    cfg = preset("qwen2.5-7b")
    p1, p8 = C.plan(cfg, tp=1), C.plan(cfg, tp=8)
    assert p8.weights < p1.weights / 3 and p8.kv <= p1.kv
    moe = preset("qwen3-30b-a3b")
    e1, e8 = C.plan(moe, "q8_0", ep=8), C.plan(moe, "q8_0", ep=8, tp=1)
    assert e8.weights == e1.weights
    assert C.plan(moe, "q8_0").weights > 4 * e8.weights


def test_fit_refusal_and_context_autosize():
    cfg = preset("qwen2.5-32b")
    with pytest.raises(C.FitError, match="largest"):
        C.check_fits(C.plan(cfg, "q4_k_m", max_context=32768, batch=64), 80 * 2**30)
    ctx = C.max_context(cfg, 180 * 2**30, batch=8)
    assert ctx % 16 == 0 and 16 <= ctx <= cfg.max_context
    assert C.plan(cfg, max_context=ctx, batch=8).total <= 180 * 2**30
    with pytest.raises(C.FitError):
        C.max_context(cfg, 10 * 2**30, batch=8)


def test_roofline_decode_prefill_and_link():
    cfg = preset("qwen2.5-7b")
    pk = R.Peaks(6548.8, 1638.8, 1400.6, 770.0, 126 * 2**20, "measured")
    d1 = R.decode_step(cfg, 1, 2048, peaks=pk)
    assert d1.bound == "memory" and 0.5e-3 < d1.time_s < 1.0e-3
    # shared 8192-token prefix: its pages are read once per step, not once per sequence
    shared = R.decode_step(cfg, 5, 9000, shared_prefix=8192, peaks=pk)
    private = R.decode_step(cfg, 5, 9000, shared_prefix=0, peaks=pk)
    assert shared.bytes < private.bytes
    pf = R.prefill(cfg, 4096, peaks=pk)
    assert pf.bound == "compute" and pf.flops > 2 * 4096 * 6e9
    tp8 = R.collective(cfg, 5, 8, peaks=pk)
    assert tp8.bound == "link" and tp8.bytes == 0 and tp8.time_s > 0
    assert R.fraction(2 * d1.time_s, d1) == pytest.approx(0.5)


def test_measured_peaks_file_is_read(tmp_path):
    f = tmp_path / "peaks.json"
    f.write_text('{"hbm_gbs": 6000, "bf16_tflops": 1500, "bf16_tflops_sustained": 1300}')
    pk = R.load_peaks(str(f))
    assert pk.hbm_gbs == 6000 and pk.source == "measured"
    assert R.load_peaks(str(tmp_path / "missing.json")).source == "nominal B200"


def test_kv_residency_split_spills_cold_tokens_to_the_host():
    from fak_b200.capacity import PAGE_TOKENS, kv_residency_split
    bpt = 1000
    s = kv_residency_split(10_000, bpt, device_free=50 * PAGE_TOKENS * bpt + 999, host_free=10 ** 9)
    assert s.hot_tokens == 50 * PAGE_TOKENS and s.tokens == 10_000 and s.cold_bytes == s.cold_tokens * bpt
    # everything fits on the device: nothing spills
    assert kv_residency_split(100, bpt, 10 ** 9, 10 ** 9).cold_tokens == 0
    # no host room: device-only sizing, never smaller
    only = kv_residency_split(10_000, bpt, 20 * PAGE_TOKENS * bpt, 0)
    assert only.hot_tokens == 20 * PAGE_TOKENS and only.cold_tokens == 0
    # host room caps the spill
    assert kv_residency_split(10_000, bpt, 0, 1234 * bpt).cold_tokens == 1234
    # fail-open on missing geometry
    assert kv_residency_split(0, bpt, 1, 1).tokens == 0 and kv_residency_split(10, 0, 1, 1).tokens == 0


def test_kv_precision_tiers():
    from fak_b200.capacity import kv_bytes_per_token, parse_kv_precision, select_kv_precision
    cfg = preset("qwen2.5-7b")
    bf16 = kv_bytes_per_token(cfg, 1, "bf16")
    assert bf16 == 28 * 2 * 4 * 128 * 2
    assert kv_bytes_per_token(cfg, 1, "q8") == int(math.ceil(bf16 / 2 * 34 / 32))
    assert bf16 / 2 < kv_bytes_per_token(cfg, 1, "fp8") < kv_bytes_per_token(cfg, 1, "q8")
    assert parse_kv_precision("") == "bf16" and parse_kv_precision("Q8_0") == "q8"
    with pytest.raises(ValueError):
        parse_kv_precision("int4")
    budget = 1000 * bf16
    assert select_kv_precision(cfg, 1000, budget) == "bf16"
    assert select_kv_precision(cfg, 1900, budget) == "fp8"
    with pytest.raises(ValueError):
        select_kv_precision(cfg, 2100, budget)
    # the plan's KV line follows the tier
    from fak_b200.capacity import plan
    assert plan(cfg, kv_precision="fp8").kv < plan(cfg).kv
