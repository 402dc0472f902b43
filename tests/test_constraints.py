"""Decode constraints: logit bias clamp, static / per-step masks, JSON prefix mask (CPU)."""
import json

import pytest
import torch

from fak_b200.engine import constraints as C
from fak_b200.engine.sampling import SamplingParams, sample_row


def test_bias_clamped_and_mask_wins(monkeypatch):
    row = torch.zeros(8)
    assert sample_row(row, SamplingParams(logit_bias={3: 5.0}), []) == 3
    biased = C.apply_constraint(row, None, {2: 1e6, 99: 1.0}, [])
    assert biased[2] == C.LOGIT_BIAS_CLAMP and biased.numel() == 8  # out-of-vocab entries ignored
    mask = C.AllowedSetMask([5, 6])
    sp = SamplingParams(mask=mask, logit_bias={2: 100.0})
    monkeypatch.delenv("FAK_NATIVE_GUIDED_DECODE", raising=False)
    assert sp.mask is not None and sample_row(row, sp, []) == 2      # mask dormant: bias decides
    monkeypatch.setenv("FAK_NATIVE_GUIDED_DECODE", "1")
    assert not sp.greedy and sample_row(row, sp, []) in (5, 6)      # mask beats any bias


def test_step_mask(monkeypatch):
    monkeypatch.setenv("FAK_NATIVE_GUIDED_DECODE", "1")
    m = C.StepMask([[1], None, [4]])
    row = torch.zeros(6)
    assert sample_row(row, SamplingParams(mask=m), []) == 1
    assert m.allowed([1], 6) is None
    assert sample_row(row, SamplingParams(mask=m), [1, 0]) == 4
    assert m.allowed([1, 0, 4], 6) is None


@pytest.mark.parametrize("text,ok", [
    ('{"a": [1, -2.5e-3, true, null], "b": {"c": "x\\u00e9"}}', True), ("[]", True), ("{}", True),
    ("[1,]", False), ('{"a" 1}', False), ("01", False), ('{"a":1}}', False), ("[1 2]", False)])
def test_json_automaton(text, ok):
    st = C._Json()
    good = all(st.feed(ch) for ch in text)
    assert good == ok
    if ok:
        assert st.complete()


def test_json_mask_generates_valid_json(monkeypatch):
    """Greedy decoding of random logits under the JSON mask always yields parseable JSON."""
    monkeypatch.setenv("FAK_NATIVE_GUIDED_DECODE", "1")
    vocab = ['{', '}', '[', ']', '"', ':', ',', ' ', 'a', 'bc', '1', '2.', '5', 'true', 'nul', 'l', '\\', '{"k":',
             '"]', 'x']
    eos = len(vocab)
    mask = C.JsonMask(lambda t: vocab[t] if t < len(vocab) else "", len(vocab) + 1, eos)
    g = torch.Generator().manual_seed(0)
    for trial in range(20):
        out = []
        for _ in range(40):
            row = torch.randn(len(vocab) + 1, generator=g)
            row[eos] += 2.0  # prefer stopping once allowed
            t = sample_row(row, SamplingParams(mask=mask), out)
            if t == eos:
                break
            out.append(t)
        text = "".join(vocab[t] for t in out)
        st = mask._state(out)
        assert st is not None, text
        if t == eos:
            json.loads(text)
