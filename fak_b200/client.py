"""Python client for a fak-b200 gateway (or any OpenAI-compatible server).

``FakClient(base_url)`` wraps the HTTP surface: chat completions (whole or streamed as token
deltas), text completions, Anthropic-style messages, embeddings, models, health, and the agent-kernel
routes (tool-call adjudication, decision journal, policy reload, stats).  Transport is ``httpx``
(any object with ``get`` / ``post`` / ``stream`` of the same shape can be injected, e.g. a FastAPI
``TestClient``).

Reference: the public SDK (pkg/fakclient/client.go) and ABI types (pkg/abi/abi.go).
"""
from __future__ import annotations

import json
from typing import Iterator


class FakError(RuntimeError):
    def __init__(self, status: int, body: str):
        super().__init__(f"HTTP {status}: {body[:500]}")
        self.status = status
        self.body = body


class FakClient:
    def __init__(self, base_url: str = "http://127.0.0.1:8000", api_key: str = "", timeout: float = 600.0,
                 http=None):
        self.base = base_url.rstrip("/")
        self.headers = {"content-type": "application/json"}
        if api_key:
            self.headers["authorization"] = f"Bearer {api_key}"
        if http is None:
            import httpx
            http = httpx.Client(timeout=timeout)
        self.http = http

    # ---- plumbing --------------------------------------------------------------------------
    def _url(self, path: str) -> str:
        return self.base + path if self.base else path

    def _check(self, r):
        if r.status_code >= 400:
            raise FakError(r.status_code, r.text)
        return r

    def _post(self, path: str, body: dict) -> dict:
        return self._check(self.http.post(self._url(path), json=body, headers=self.headers)).json()

    def _get(self, path: str, **params) -> dict:
        return self._check(self.http.get(self._url(path), params=params or None, headers=self.headers)).json()

    def _sse(self, path: str, body: dict) -> Iterator[tuple[str | None, dict]]:
        """(event name, data) for each server-sent event until [DONE]."""
        with self.http.stream("POST", self._url(path), json=body, headers=self.headers) as r:
            if r.status_code >= 400:
                r.read()
                raise FakError(r.status_code, r.text)
            event = None
            for line in r.iter_lines():
                if isinstance(line, bytes):
                    line = line.decode()
                if not line:
                    event = None
                    continue
                if line.startswith("event:"):
                    event = line[6:].strip()
                elif line.startswith("data:"):
                    data = line[5:].strip()
                    if data == "[DONE]":
                        return
                    yield event, json.loads(data)

    # ---- OpenAI / Anthropic surface ---------------------------------------------------------
    def health(self) -> dict:
        return self._get("/healthz")

    def models(self) -> list[str]:
        return [m["id"] for m in self._get("/v1/models")["data"]]

    def chat(self, messages: list[dict], model: str = "fak", max_tokens: int = 256, **kw) -> dict:
        return self._post("/v1/chat/completions", dict(model=model, messages=messages, max_tokens=max_tokens, **kw))

    def chat_text(self, messages: list[dict], **kw) -> str:
        return self.chat(messages, **kw)["choices"][0]["message"].get("content") or ""

    def stream_chat(self, messages: list[dict], model: str = "fak", max_tokens: int = 256, **kw) -> Iterator[str]:
        """Content deltas of a streamed chat completion."""
        body = dict(model=model, messages=messages, max_tokens=max_tokens, stream=True, **kw)
        for _, d in self._sse("/v1/chat/completions", body):
            for ch in d.get("choices", []):
                c = (ch.get("delta") or {}).get("content")
                if c:
                    yield c

    def complete(self, prompt: str, model: str = "fak", max_tokens: int = 128, **kw) -> str:
        r = self._post("/v1/completions", dict(model=model, prompt=prompt, max_tokens=max_tokens, **kw))
        return r["choices"][0]["text"]

    def messages(self, messages: list[dict], model: str = "fak", max_tokens: int = 256, **kw) -> dict:
        return self._post("/v1/messages", dict(model=model, messages=messages, max_tokens=max_tokens, **kw))

    def embeddings(self, inputs: list[str] | str, model: str = "fak") -> list[list[float]]:
        r = self._post("/v1/embeddings", {"model": model, "input": inputs})
        return [d["embedding"] for d in r["data"]]

    # ---- agent kernel ------------------------------------------------------------------------
    def adjudicate(self, name: str, arguments: dict, trace_id: str = "") -> dict:
        """Verdict of the gateway's kernel on one proposed tool call."""
        return self._post("/v1/fak/adjudicate", {"name": name, "arguments": arguments, "trace_id": trace_id})

    def journal(self, n: int = 50) -> list[dict]:
        return self._get("/v1/fak/journal", n=n)["entries"]

    def set_policy(self, policy: dict) -> dict:
        return self._post("/v1/fak/policy", policy)

    def stats(self) -> dict:
        return self._get("/v1/fak/stats")
