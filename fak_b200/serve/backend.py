"""Model backends behind the gateway.

``EngineBackend``   the GPU engine; one background thread drives ``Engine.step()`` while
                    request threads wait on per-request token queues (continuous batching:
                    concurrent requests decode together).
``ReferenceBackend`` the fp32 PyTorch reference on CPU (tests, tiny models, no GPU).
``UpstreamBackend`` proxy mode: forward to an upstream OpenAI-compatible server and only
                    adjudicate what comes back (the reference's gateway-in-front-of-a-model role).
"""
from __future__ import annotations

import json
import queue
import threading
import time
from typing import Iterator

from ..engine.sampling import SamplingParams

_DONE = object()


class EngineBackend:
    def __init__(self, engine, tokenizer, name: str = "fak-b200"):
        self.engine = engine
        self.tok = tokenizer
        self.name = name
        self._lock = threading.Lock()
        self._wake = threading.Event()
        self._stop = False
        self._thread = threading.Thread(target=self._loop, name="fak-engine", daemon=True)
        self._thread.start()

    def _loop(self) -> None:
        while not self._stop:
            with self._lock:
                busy = self.engine.has_work()
                if busy:
                    self.engine.step()
            if not busy:
                self._wake.wait(0.05)
                self._wake.clear()

    def generate(self, prompt_ids: list[int], max_tokens: int, sampling: SamplingParams,
                 stop_ids=()) -> Iterator[int]:
        q: queue.Queue = queue.Queue()

        def on_token(t: int) -> None:
            q.put(t)

        with self._lock:
            req = self.engine.add_request(prompt_ids, max_tokens, sampling, stop_ids, on_token=on_token)
        self._wake.set()
        n = 0
        while True:
            try:
                t = q.get(timeout=0.02)
            except queue.Empty:
                if req.finished and q.empty():
                    break
                continue
            n += 1
            yield t
            if req.finished and q.empty():
                break
        self.last_request = req

    def close(self) -> None:
        self._stop = True
        self._wake.set()
        self._thread.join(timeout=5)


class CachelessModel:
    """Adapts a whole-sequence model (``forward(ids) -> logits``, e.g. GlmDsaReference or
    Gemma4Reference) to the incremental ``forward(ids, start_pos, kv)`` the reference backend
    calls: ``kv`` keeps the token history and every call re-runs the full sequence, returning the
    logits of the new tokens (quadratic in length; a correctness path, not a fast one)."""

    def __init__(self, model):
        self.model = model

    def forward(self, ids, start_pos: int = 0, kv: list | None = None):
        import torch
        ids = torch.as_tensor(ids, dtype=torch.long).reshape(-1)
        hist = kv if kv is not None else []
        if len(hist) != start_pos:
            raise ValueError(f"history holds {len(hist)} tokens, call starts at {start_pos}")
        hist.extend(int(t) for t in ids)
        return self.model.forward(torch.tensor(hist))[-ids.numel():]


class ReferenceBackend:
    def __init__(self, model, tokenizer, name: str = "fak-b200-reference"):
        import torch  # noqa: F401
        self.model = model
        self.tok = tokenizer
        self.name = name
        self._lock = threading.Lock()

    def generate(self, prompt_ids: list[int], max_tokens: int, sampling: SamplingParams,
                 stop_ids=()) -> Iterator[int]:
        import torch
        from ..engine.sampling import sample_row
        with self._lock, torch.no_grad():
            kv: list = []
            logits = self.model.forward(torch.tensor(prompt_ids), 0, kv)[-1]
            pos = len(prompt_ids)
            out: list[int] = []
            for _ in range(max_tokens):
                t = sample_row(logits, sampling, out)
                out.append(t)
                yield t
                if t in stop_ids:
                    break
                logits = self.model.forward(torch.tensor([t]), pos, kv)[-1]
                pos += 1


class UpstreamBackend:
    """Forwards chat requests to an upstream OpenAI-compatible endpoint (no local model)."""

    def __init__(self, base_url: str, api_key: str = "", name: str = "upstream", timeout: float = 600.0):
        self.base = base_url.rstrip("/")
        self.key = api_key
        self.name = name
        self.timeout = timeout
        self.tok = None

    def chat(self, body: dict) -> dict:
        import httpx
        headers = {"content-type": "application/json"}
        if self.key:
            headers["authorization"] = f"Bearer {self.key}"
        b = dict(body, stream=False)
        r = httpx.post(self.base + "/v1/chat/completions", json=b, headers=headers, timeout=self.timeout)
        r.raise_for_status()
        return r.json()
