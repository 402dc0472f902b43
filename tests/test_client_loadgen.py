"""Public client SDK and the load generator against the in-process gateway (CPU); speculative
decoding expectation arithmetic."""
import math

import pytest

fastapi = pytest.importorskip("fastapi")
from fastapi.testclient import TestClient  # noqa: E402

from fak_b200.agentkernel import Kernel  # noqa: E402
from fak_b200.client import FakClient, FakError  # noqa: E402
from fak_b200.config import preset  # noqa: E402
from fak_b200.engine.specmath import AcceptanceMeter, best_k, expected_tokens, speedup  # noqa: E402
from fak_b200.gguf import open_gguf  # noqa: E402
from fak_b200.gguf.synth import write_synthetic_gguf  # noqa: E402
from fak_b200.serve import Gateway, create_app  # noqa: E402
from fak_b200.tokenizer import Tokenizer  # noqa: E402


class _Echo:
    def __init__(self, tok):
        self.tok, self.name = tok, "echo"

    def generate(self, ids, max_tokens, sampling, stop_ids=()):
        for t in self.tok.encode("hello there friend")[:max_tokens]:
            yield t
        yield self.tok.token_to_id["<|im_end|>"]


@pytest.fixture(scope="module")
def client(tmp_path_factory):
    p = str(tmp_path_factory.mktemp("m") / "t.gguf")
    write_synthetic_gguf(p, preset("tiny-qwen2"), "f32", seed=2)
    tok = Tokenizer.from_gguf_metadata(open_gguf(p).metadata)
    gw = Gateway(_Echo(tok), Kernel())
    return FakClient("", http=TestClient(create_app(gw)))


def test_client_surface(client):
    assert client.health()
    assert client.models()
    msgs = [{"role": "user", "content": "hi"}]
    assert client.chat_text(msgs) == "hello there friend"
    assert "".join(client.stream_chat(msgs)) == "hello there friend"
    assert client.complete("x")
    v = client.adjudicate("Bash", {"command": "sudo rm -rf /"})
    assert v["kind"] == "DENY" and v["reason"] == "POLICY_BLOCK"
    assert client.adjudicate("Read", {"path": "a.txt"})["kind"] == "ALLOW"
    assert len(client.journal(10)) >= 2
    assert "kernel" in client.stats()
    with pytest.raises(FakError):
        client.set_policy({"schema": "nope", "allow": 5})


def test_loadgen_levels(client):
    from fak_b200.benchmarks.loadgen import run_level
    r = run_level(lambda: client, 2, 6, "go", 8)
    assert r["requests"] == 6 and r["errors"] == 0 and r["ttft_ms_p50"] is not None and r["deltas_per_s"] > 0


def test_spec_expectation():
    assert expected_tokens(4, 1.0) == 5 and expected_tokens(4, 0.0) == 1
    assert math.isclose(expected_tokens(3, 0.5), 1 + 0.5 + 0.25 + 0.125)
    k, s = best_k(0.8, draft_cost=0.1)
    assert k > 0 and s == pytest.approx(speedup(k, 0.8, 0.1)) and s > 1
    assert best_k(0.0, draft_cost=0.1)[0] == 0
    m = AcceptanceMeter()
    m.observe(4, 3)
    m.observe(4, 1)
    assert m.rate == 0.5 and m.tokens_per_step == 3.0
    with pytest.raises(ValueError):
        m.observe(2, 3)
