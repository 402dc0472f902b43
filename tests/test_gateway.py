"""Gateway routes, streaming, tool-call adjudication, upstream proxy (CPU, fake + reference backends)."""
import json

import pytest

fastapi = pytest.importorskip("fastapi")
from fastapi.testclient import TestClient  # noqa: E402

from fak_b200.agentkernel import Kernel, policy_from_dict  # noqa: E402
from fak_b200.config import preset  # noqa: E402
from fak_b200.gguf import open_gguf  # noqa: E402
from fak_b200.gguf.synth import write_synthetic_gguf  # noqa: E402
from fak_b200.serve import Gateway, ReferenceBackend, create_app  # noqa: E402
from fak_b200.serve.chat import extract_tool_calls, render_chatml  # noqa: E402
from fak_b200.tokenizer import Tokenizer  # noqa: E402


@pytest.fixture(scope="module")
def tok(tmp_path_factory):
    p = str(tmp_path_factory.mktemp("m") / "t.gguf")
    write_synthetic_gguf(p, preset("tiny-qwen2"), "f32", seed=2)
    return p, Tokenizer.from_gguf_metadata(open_gguf(p).metadata)


class ScriptedBackend:
    """Emits a fixed completion (tokenized), standing in for a model that proposes tool calls."""

    def __init__(self, tok, text):
        self.tok, self.text, self.name = tok, text, "scripted"

    def generate(self, ids, max_tokens, sampling, stop_ids=()):
        for t in self.tok.encode(self.text)[:max_tokens]:
            yield t
        yield self.tok.token_to_id["<|im_end|>"]


def _client(tok, text, policy=None):
    k = Kernel(policy_from_dict(policy) if policy else None)
    gw = Gateway(ScriptedBackend(tok, text), k)
    return TestClient(create_app(gw)), gw


CALLS = ('ok <tool_call>{"name": "Read", "arguments": {"path": "a.txt"}}</tool_call>'
         '<tool_call>{"name": "Bash", "arguments": {"command": "sudo rm -rf /"}}</tool_call>')


def test_render_and_extract():
    s = render_chatml([{"role": "user", "content": "hi"}], tools=[{"type": "function", "function": {
        "name": "Read", "parameters": {"type": "object"}}}])
    assert "<tools>" in s and s.endswith("<|im_start|>assistant\n")
    plain, calls = extract_tool_calls(CALLS)
    assert plain == "ok" and [c["name"] for c in calls] == ["Read", "Bash"]


def test_chat_completion_adjudicates_tool_calls(tok):
    _, t = tok
    c, gw = _client(t, CALLS)
    r = c.post("/v1/chat/completions", json={"model": "x", "messages": [{"role": "user", "content": "go"}]}).json()
    msg = r["choices"][0]["message"]
    assert [tc["function"]["name"] for tc in msg["tool_calls"]] == ["Read"]
    assert "refused: POLICY_BLOCK" in msg["content"]
    assert r["choices"][0]["finish_reason"] == "tool_calls"
    j = c.get("/v1/fak/journal").json()
    assert j["chain_ok"] and len(j["entries"]) == 2
    assert "fak_kernel_verdicts_total" in c.get("/metrics").text


def test_chat_stream_holds_tool_calls(tok):
    _, t = tok
    c, _ = _client(t, CALLS)
    with c.stream("POST", "/v1/chat/completions", json={"messages": [{"role": "user", "content": "x"}],
                                                        "stream": True}) as r:
        lines = [l for l in r.iter_lines() if l.startswith("data: ")]
    assert lines[-1] == "data: [DONE]"
    chunks = [json.loads(l[6:]) for l in lines[:-1]]
    content = "".join(ch["choices"][0]["delta"].get("content") or "" for ch in chunks)
    assert "<tool_call>" not in content and "refused" in content
    tcs = [ch["choices"][0]["delta"]["tool_calls"] for ch in chunks if "tool_calls" in ch["choices"][0]["delta"]]
    assert len(tcs) == 1 and tcs[0][0]["function"]["name"] == "Read"


def test_anthropic_messages_and_stream(tok):
    _, t = tok
    c, _ = _client(t, CALLS)
    r = c.post("/v1/messages", json={"model": "m", "max_tokens": 200, "system": "s",
                                     "messages": [{"role": "user", "content": [{"type": "text", "text": "go"}]}]}).json()
    kinds = [b["type"] for b in r["content"]]
    assert kinds == ["text", "tool_use"] and r["stop_reason"] == "tool_use"
    with c.stream("POST", "/v1/messages", json={"max_tokens": 200, "stream": True,
                                                "messages": [{"role": "user", "content": "go"}]}) as s:
        events = [l[7:] for l in s.iter_lines() if l.startswith("event: ")]
    assert events[0] == "message_start" and events[-1] == "message_stop"


def test_adjudicate_and_policy_reload(tok):
    _, t = tok
    c, _ = _client(t, "hi")
    assert c.post("/v1/fak/adjudicate", json={"tool": "launch", "args": {}}).json()["reason"] == "DEFAULT_DENY"
    assert c.post("/v1/fak/policy", json={"allow": ["launch"]}).json()["ok"]
    assert c.post("/v1/fak/adjudicate", json={"tool": "launch", "args": {}}).json()["kind"] == "ALLOW"
    assert c.post("/v1/fak/policy", json={"bogus": 1}).status_code == 400


def test_reference_backend_end_to_end(tok):
    path, t = tok
    from fak_b200.models.reference import ReferenceModel
    gw = Gateway(ReferenceBackend(ReferenceModel.from_gguf(path), t))
    c = TestClient(create_app(gw))
    r = c.post("/v1/completions", json={"prompt": "hello", "max_tokens": 5}).json()
    assert r["usage"]["completion_tokens"] >= 1
    r = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}], "max_tokens": 4})
    assert r.status_code == 200 and r.json()["usage"]["prompt_tokens"] > 5


def test_metrics_expose_tpot_and_engine_stats(tok):
    _, t = tok

    class FakeEngine:
        stats = {"prefill_tokens_avoided": 4096, "decode_tokens": 7, "spec_proposed": 8, "spec_accepted": 6}
        waiting, prefilling, running = [1], [], [1, 2]

    b = ScriptedBackend(t, "hello there, general")
    b.engine = FakeEngine()
    gw = Gateway(b, Kernel())
    c = TestClient(create_app(gw))
    c.post("/v1/chat/completions", json={"model": "x", "messages": [{"role": "user", "content": "go"}]})
    text = c.get("/metrics").text
    assert "fak_gateway_tpot_seconds_count" in text
    assert 'fak_engine_stat{stat="prefill_tokens_avoided"} 4096.0' in text
    assert 'fak_engine_stat{stat="spec_acceptance"} 0.75' in text
    assert 'fak_engine_stat{stat="requests_running"} 2.0' in text


def test_response_format_json_mask_is_built_from_the_vocabulary(tok, monkeypatch):
    _, t = tok
    gw = Gateway(ScriptedBackend(t, '{"a": 1}'), Kernel())
    from fak_b200.serve.gateway import _sampling
    sp = _sampling({"response_format": {"type": "json_object"}}, gw._json_mask)
    assert sp.mask is not None and sp.mask is gw._json_mask()  # built once
    monkeypatch.setenv("FAK_NATIVE_GUIDED_DECODE", "1")
    assert not sp.greedy
    ok = sp.mask.allowed([], t.vocab_size)
    brace = t.token_to_id.get("{")
    assert brace is None or bool(ok[brace])
