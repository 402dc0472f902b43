"""OpenAI- and Anthropic-compatible HTTP gateway with the agent-kernel floor in the loop.

Routes (reference surface: internal/gateway/http.go:54-131):
  POST /v1/chat/completions   OpenAI chat (SSE streaming with ``stream: true``)
  POST /v1/completions        OpenAI text completion
  POST /v1/messages           Anthropic messages (SSE event stream with ``stream: true``)
  POST /v1/embeddings         mean-pooled final hidden state
  GET  /v1/models, /healthz, /metrics (Prometheus)
  POST /v1/fak/adjudicate     run one tool call through the floor
  GET  /v1/fak/journal        tail of the hash-chained decision journal (+ chain check)
  POST /v1/fak/policy         hot-reload a validated policy manifest
  GET  /v1/fak/stats          kernel + engine counters (radix reuse, TTFT, verdicts)
  + the Responses / count_tokens / moderations / Gemini / syscall / admit / MCP / A2A surfaces and
    the admission and autoscaler views of ``serve/surfaces.py``

With an ``AdmissionController`` every generating request holds an admission lease (priority from the
``X-Fak-Priority`` header or the body's ``priority``; a full waiting queue answers 429, a denied
tenant 403).  Completed requests feed the autoscaler's signal window (TTFT, TPOT, goodput).

Every tool call the model proposes is adjudicated before it is returned to the client: allowed
calls pass (with redacted arguments under TRANSFORM), refused calls are removed from the
response and replaced by a refusal note the agent can read, and every decision is journaled.
"""
from __future__ import annotations

import json
import time
import uuid
from typing import Any, Iterator

from fastapi import FastAPI, HTTPException, Request
from fastapi.responses import JSONResponse, PlainTextResponse, StreamingResponse

import contextlib

from ..agentkernel import Kernel, ToolCall, VerdictKind, policy_from_dict
from ..engine.sampling import SamplingParams
from ..tokenizer import IncrementalDecoder
from .admission import AdmissionController, AdmissionError, SeqRequest
from .autoscale import PoolObjective, ServingAutoscaler, SignalWindow
from .backend import UpstreamBackend
from .chat import extract_tool_calls, render_chatml


def _sampling(body: dict, json_mask=None) -> SamplingParams:
    """Request sampling fields; ``response_format: {"type": "json_object"}`` adds the JSON mask
    (active when guided decoding is switched on, FAK_NATIVE_GUIDED_DECODE=1)."""
    rf = body.get("response_format") or {}
    mask = json_mask() if json_mask is not None and isinstance(rf, dict) and rf.get("type") in (
        "json_object", "json_schema") else None
    return SamplingParams(mask=mask, temperature=float(body.get("temperature", 0.0) or 0.0),
                          top_k=int(body.get("top_k", 0) or 0), top_p=float(body.get("top_p", 1.0) or 1.0),
                          frequency_penalty=float(body.get("frequency_penalty", 0.0) or 0.0),
                          presence_penalty=float(body.get("presence_penalty", 0.0) or 0.0),
                          logit_bias={int(k): float(v) for k, v in (body.get("logit_bias") or {}).items()} or None,
                          seed=body.get("seed"))


class Metrics:
    def __init__(self):
        from prometheus_client import CollectorRegistry, Counter, Histogram
        self.registry = CollectorRegistry()
        self.requests = Counter("fak_gateway_http_requests_total", "HTTP requests", ["route"], registry=self.registry)
        self.duration = Histogram("fak_gateway_http_request_duration_seconds", "request latency", ["route"],
                                  registry=self.registry)
        self.ttft = Histogram("fak_gateway_ttft_seconds", "time to first token", registry=self.registry,
                              buckets=(0.005, 0.01, 0.025, 0.05, 0.1, 0.25, 0.5, 1, 2.5, 5, 10))
        self.tokens = Counter("fak_gateway_completion_tokens_total", "generated tokens", registry=self.registry)
        self.prompt_tokens = Counter("fak_gateway_prompt_tokens_total", "prompt tokens", registry=self.registry)
        self.verdicts = Counter("fak_kernel_verdicts_total", "tool-call verdicts", ["kind", "reason"],
                                registry=self.registry)
        self.tpot = Histogram("fak_gateway_tpot_seconds", "time per output token after the first",
                              registry=self.registry,
                              buckets=(0.001, 0.0025, 0.005, 0.01, 0.025, 0.05, 0.1, 0.25))
        from prometheus_client import Gauge
        self.engine = Gauge("fak_engine_stat", "engine counters and gauges (scraped from the engine)", ["stat"],
                            registry=self.registry)

    def scrape_engine(self, backend) -> None:
        """Copy the local engine's counters (prefill tokens avoided, radix hit rate, KV pages, spec
        acceptance, queue depths) into gauges at scrape time."""
        eng = getattr(backend, "engine", None)
        if eng is None:
            return
        st = dict(getattr(eng, "stats", {}))
        radix = getattr(eng, "radix", None)
        if radix is not None:
            for k, v in radix.stats().items():
                st["radix_" + k] = v
        pool = getattr(eng, "pool", None)
        if pool is not None:
            st["kv_pages_free"] = pool.n_free()
        for name in ("waiting", "prefilling", "running"):
            if hasattr(eng, name):
                st["requests_" + name] = len(getattr(eng, name))
        if st.get("spec_proposed"):
            st["spec_acceptance"] = st.get("spec_accepted", 0) / st["spec_proposed"]
        for k, v in st.items():
            if isinstance(v, (int, float)):
                self.engine.labels(k).set(float(v))


class Gateway:
    def __init__(self, backend, kernel: Kernel | None = None, model_name: str | None = None,
                 default_max_tokens: int = 256, ctx_view_budget: int = 0,
                 admission: AdmissionController | None = None, objective: PoolObjective | None = None):
        self.backend = backend
        self.admission = admission
        self.objective = objective or PoolObjective()
        self.signals = SignalWindow(self.objective)
        self.autoscaler = ServingAutoscaler({"decode": self.objective})
        self.planner = None   # planned context views under a token budget (0: whole transcript)
        if ctx_view_budget > 0:
            from .ctxplan import ContextPlanner
            tok = getattr(backend, "tok", None)
            count = (lambda s: len(tok.encode(s))) if tok is not None else None
            self.planner = ContextPlanner(ctx_view_budget, count)
        self.kernel = kernel or Kernel()
        self.model_name = model_name or getattr(backend, "name", "fak-b200")
        self.default_max_tokens = default_max_tokens
        self.metrics = Metrics()
        self.tok = getattr(backend, "tok", None)
        self._json = None

    # ------------------------------------------------------------------ admission / autoscale
    def count_prompt_tokens(self, text: str) -> int:
        return len(self.tok.encode(text)) if self.tok is not None else max(1, len(text) // 4)

    @contextlib.contextmanager
    def lease(self, body: dict, route: str, priority: int | None = None):
        """Hold an admission lease around one generating request (no-op without a controller)."""
        if self.admission is None:
            yield None
            return
        msgs = body.get("messages") or []
        est = sum(len(json.dumps(m)) for m in msgs) // 4 + len(str(body.get("prompt", ""))) // 4
        toks = est + int(body.get("max_tokens") or body.get("max_completion_tokens") or self.default_max_tokens)
        pr = int(body.get("priority", 0) if priority is None else priority)
        r = SeqRequest(trace_id=f"{route}-{uuid.uuid4().hex[:16]}", priority=pr, tokens=toks)
        try:
            with self.admission.lease(r) as held:
                yield held
        except AdmissionError as e:
            raise HTTPException(e.status, str(e))

    def autoscale_decision(self, replicas: int = 1) -> dict:
        eng = getattr(self.backend, "engine", None)
        depth = len(getattr(eng, "waiting", [])) if eng is not None else 0
        if self.admission is not None:
            depth += self.admission.snapshot()["waiting"]
        kv = 0.0
        pool = getattr(eng, "pool", None)
        if pool is not None and getattr(pool, "n_pages", 0):
            kv = 1.0 - pool.n_free() / pool.n_pages
        sig = self.signals.signals(depth, kv)
        return self.autoscaler.plan("decode", int(replicas), sig).to_dict()

    def _view(self, messages: list[dict]) -> list[dict]:
        return self.planner.plan(messages).messages if self.planner is not None and messages else messages

    # ------------------------------------------------------------------ generation core
    def _stop_ids(self) -> set[int]:
        ids = set()
        if self.tok is not None:
            for s in ("<|im_end|>", "<|endoftext|>"):
                i = self.tok.token_to_id.get(s)
                if i is not None:
                    ids.add(i)
            if self.tok.eos_id is not None:
                ids.add(int(self.tok.eos_id))
        return ids

    def stream_text(self, prompt: str, max_tokens: int, sampling: SamplingParams, stop: list[str] | None = None
                    ) -> Iterator[tuple[str, dict]]:
        """Yield (text delta, info) pairs; info of the last item carries usage/finish data."""
        ids = self.tok.encode(prompt)
        self.metrics.prompt_tokens.inc(len(ids))
        stop_ids = self._stop_ids()
        dec = IncrementalDecoder(self.tok, skip_special=True)
        t0 = time.perf_counter()
        n, text, first = 0, "", None
        finish = "length"
        for t in self.backend.generate(ids, max_tokens, sampling, stop_ids):
            if first is None:
                first = time.perf_counter() - t0
                self.metrics.ttft.observe(first)
            n += 1
            if t in stop_ids:
                finish = "stop"
                break
            piece = dec.push(t)
            text += piece
            if stop:
                hit = [text.find(s) for s in stop if s and text.find(s) >= 0]
                if hit:
                    cut = min(hit)
                    piece = piece[: max(0, len(piece) - (len(text) - cut))]
                    text = text[:cut]
                    finish = "stop"
                    if piece:
                        yield piece, {}
                    break
            if piece:
                yield piece, {}
        tail = dec.flush()
        if tail and finish != "stop":
            text += tail
            yield tail, {}
        self.metrics.tokens.inc(n)
        tpot = None
        if first is not None and n > 1:
            tpot = (time.perf_counter() - t0 - first) / (n - 1)
            self.metrics.tpot.observe(tpot)
        self.signals.observe(first, tpot)
        yield "", {"prompt_tokens": len(ids), "completion_tokens": n, "finish_reason": finish,
                   "ttft_s": first, "text": text}

    def adjudicate_calls(self, calls: list[dict], trace_id: str = "") -> tuple[list[dict], list[str]]:
        allowed, notes = [], []
        for c in calls:
            tc = ToolCall(tool=c["name"], args=c["arguments"] if isinstance(c["arguments"], dict) else {},
                          trace_id=trace_id)
            v = self.kernel.decide(tc)
            self.metrics.verdicts.labels(v.kind.name, v.reason.name).inc()
            if v.allowed:
                args = v.new_args if v.kind == VerdictKind.TRANSFORM and v.new_args is not None else c["arguments"]
                allowed.append(dict(c, arguments=args))
            else:
                notes.append(f"[fak] tool call `{c['name']}` refused: {v.reason.name}"
                             + (f" ({v.claim})" if v.claim else ""))
        return allowed, notes

    def _json_mask(self):
        """JSON-prefix token mask over this tokenizer's vocabulary (built once)."""
        if self.tok is None:
            return None
        if self._json is None:
            from ..engine.constraints import JsonMask
            self._json = JsonMask(lambda t: self.tok.decode([t]), self.tok.vocab_size, self.tok.eos_id)
        return self._json

    # ------------------------------------------------------------------ OpenAI
    def chat_completion(self, body: dict) -> dict:
        rid = "chatcmpl-" + uuid.uuid4().hex[:24]
        if isinstance(self.backend, UpstreamBackend):
            resp = self.backend.chat(body)
            for ch in resp.get("choices", []):
                msg = ch.get("message", {})
                calls = [{"id": tc.get("id"), "name": tc["function"]["name"],
                          "arguments": json.loads(tc["function"].get("arguments") or "{}")}
                         for tc in msg.get("tool_calls") or []]
                allowed, notes = self.adjudicate_calls(calls, rid)
                msg["tool_calls"] = [{"id": c["id"], "type": "function",
                                      "function": {"name": c["name"], "arguments": json.dumps(c["arguments"])}}
                                     for c in allowed] or None
                if notes:
                    msg["content"] = ((msg.get("content") or "") + "\n" + "\n".join(notes)).strip()
            return resp
        self.kernel.preflight.register_openai_tools(body.get("tools"))   # schemas for the pre-flight rungs
        self.kernel.grammar.register_openai_tools(body.get("tools"))     # and the tools' argument grammars
        prompt = render_chatml(self._view(body.get("messages", [])), body.get("tools"))
        info = {}
        text = ""
        stop = body.get("stop")
        stop = [stop] if isinstance(stop, str) else stop
        for piece, inf in self.stream_text(prompt, int(body.get("max_tokens") or body.get("max_completion_tokens")
                                                       or self.default_max_tokens), _sampling(body, self._json_mask), stop):
            text += piece
            info = inf or info
        plain, calls = extract_tool_calls(text)
        allowed, notes = self.adjudicate_calls(calls, rid)
        content = "\n".join([plain] + notes).strip() if notes else plain
        msg: dict[str, Any] = {"role": "assistant", "content": content or None}
        if allowed:
            msg["tool_calls"] = [{"id": c["id"], "type": "function",
                                  "function": {"name": c["name"], "arguments": json.dumps(c["arguments"])}}
                                 for c in allowed]
        finish = "tool_calls" if allowed else info.get("finish_reason", "stop")
        return {"id": rid, "object": "chat.completion", "created": int(time.time()), "model": self.model_name,
                "choices": [{"index": 0, "message": msg, "finish_reason": finish}],
                "usage": {"prompt_tokens": info.get("prompt_tokens", 0),
                          "completion_tokens": info.get("completion_tokens", 0),
                          "total_tokens": info.get("prompt_tokens", 0) + info.get("completion_tokens", 0)}}

    def chat_completion_stream(self, body: dict) -> Iterator[str]:
        rid = "chatcmpl-" + uuid.uuid4().hex[:24]
        created = int(time.time())

        def chunk(delta: dict, finish=None) -> str:
            return "data: " + json.dumps({"id": rid, "object": "chat.completion.chunk", "created": created,
                                          "model": self.model_name,
                                          "choices": [{"index": 0, "delta": delta, "finish_reason": finish}]}) + "\n\n"

        yield chunk({"role": "assistant"})
        self.kernel.preflight.register_openai_tools(body.get("tools"))   # schemas for the pre-flight rungs
        self.kernel.grammar.register_openai_tools(body.get("tools"))     # and the tools' argument grammars
        prompt = render_chatml(self._view(body.get("messages", [])), body.get("tools"))
        text, info, held = "", {}, ""
        for piece, inf in self.stream_text(prompt, int(body.get("max_tokens") or self.default_max_tokens),
                                           _sampling(body, self._json_mask), None):
            info = inf or info
            if not piece:
                continue
            text += piece
            # hold back anything that may be part of a <tool_call> block until it is adjudicated
            held += piece
            out = ""
            while held:
                i = held.find("<")
                if i < 0:
                    out, held = out + held, ""
                    break
                out, held = out + held[:i], held[i:]
                if held.startswith("<tool_call>") or "<tool_call>".startswith(held):
                    break  # a tool call (or the start of one): keep it until the end
                out, held = out + held[0], held[1:]
            if out:
                yield chunk({"content": out})
        plain_tail, calls = extract_tool_calls(held)
        if plain_tail:
            yield chunk({"content": plain_tail})
        allowed, notes = self.adjudicate_calls(calls, rid)
        if notes:
            yield chunk({"content": "\n" + "\n".join(notes)})
        if allowed:
            yield chunk({"tool_calls": [{"index": i, "id": c["id"], "type": "function",
                                         "function": {"name": c["name"], "arguments": json.dumps(c["arguments"])}}
                                        for i, c in enumerate(allowed)]})
        yield chunk({}, "tool_calls" if allowed else info.get("finish_reason", "stop"))
        yield "data: [DONE]\n\n"

    def completion(self, body: dict) -> dict:
        prompt = body.get("prompt", "")
        if isinstance(prompt, list):
            prompt = prompt[0] if prompt else ""
        text, info = "", {}
        stop = body.get("stop")
        stop = [stop] if isinstance(stop, str) else stop
        for piece, inf in self.stream_text(prompt, int(body.get("max_tokens") or 16), _sampling(body, self._json_mask), stop):
            text += piece
            info = inf or info
        return {"id": "cmpl-" + uuid.uuid4().hex[:24], "object": "text_completion", "created": int(time.time()),
                "model": self.model_name,
                "choices": [{"index": 0, "text": text, "finish_reason": info.get("finish_reason", "stop")}],
                "usage": {"prompt_tokens": info.get("prompt_tokens", 0),
                          "completion_tokens": info.get("completion_tokens", 0)}}

    # ------------------------------------------------------------------ Anthropic
    def _anthropic_prompt(self, body: dict) -> str:
        return render_chatml(body.get("messages", []), body.get("tools"), system=body.get("system"))

    def messages(self, body: dict) -> dict:
        mid = "msg_" + uuid.uuid4().hex[:24]
        text, info = "", {}
        for piece, inf in self.stream_text(self._anthropic_prompt(body), int(body.get("max_tokens") or 256),
                                           _sampling(body, self._json_mask), body.get("stop_sequences")):
            text += piece
            info = inf or info
        plain, calls = extract_tool_calls(text)
        allowed, notes = self.adjudicate_calls(calls, mid)
        content: list[dict] = []
        body_text = "\n".join([plain] + notes).strip() if notes else plain
        if body_text:
            content.append({"type": "text", "text": body_text})
        for c in allowed:
            content.append({"type": "tool_use", "id": "toolu_" + c["id"][5:], "name": c["name"], "input": c["arguments"]})
        stop_reason = "tool_use" if allowed else ("max_tokens" if info.get("finish_reason") == "length" else "end_turn")
        return {"id": mid, "type": "message", "role": "assistant", "model": body.get("model", self.model_name),
                "content": content, "stop_reason": stop_reason, "stop_sequence": None,
                "usage": {"input_tokens": info.get("prompt_tokens", 0),
                          "output_tokens": info.get("completion_tokens", 0)}}

    def messages_stream(self, body: dict) -> Iterator[str]:
        def ev(name: str, data: dict) -> str:
            return f"event: {name}\ndata: {json.dumps(data)}\n\n"

        msg = self.messages(body)  # generation is adjudicated as a whole before tool blocks stream
        yield ev("message_start", {"type": "message_start",
                                   "message": dict(msg, content=[], stop_reason=None,
                                                   usage={"input_tokens": msg["usage"]["input_tokens"],
                                                          "output_tokens": 0})})
        for i, block in enumerate(msg["content"]):
            if block["type"] == "text":
                yield ev("content_block_start", {"type": "content_block_start", "index": i,
                                                 "content_block": {"type": "text", "text": ""}})
                yield ev("content_block_delta", {"type": "content_block_delta", "index": i,
                                                 "delta": {"type": "text_delta", "text": block["text"]}})
            else:
                yield ev("content_block_start", {"type": "content_block_start", "index": i,
                                                 "content_block": {"type": "tool_use", "id": block["id"],
                                                                   "name": block["name"], "input": {}}})
                yield ev("content_block_delta", {"type": "content_block_delta", "index": i,
                                                 "delta": {"type": "input_json_delta",
                                                           "partial_json": json.dumps(block["input"])}})
            yield ev("content_block_stop", {"type": "content_block_stop", "index": i})
        yield ev("message_delta", {"type": "message_delta", "delta": {"stop_reason": msg["stop_reason"]},
                                   "usage": {"output_tokens": msg["usage"]["output_tokens"]}})
        yield ev("message_stop", {"type": "message_stop"})

    # ------------------------------------------------------------------ embeddings
    def embeddings(self, body: dict) -> dict:
        inp = body.get("input", "")
        texts = [inp] if isinstance(inp, str) else list(inp)
        embed = getattr(self.backend, "embed", None)
        if embed is None:
            raise NotImplementedError("this backend has no embedding path")
        data = [{"object": "embedding", "index": i, "embedding": embed(self.tok.encode(t))} for i, t in enumerate(texts)]
        return {"object": "list", "data": data, "model": self.model_name}


def create_app(gw: Gateway) -> FastAPI:
    app = FastAPI(title="fak-b200 gateway")

    def timed(route: str):
        gw.metrics.requests.labels(route).inc()
        return gw.metrics.duration.labels(route).time()

    @app.get("/healthz")
    def healthz():
        return {"ok": True, "model": gw.model_name}

    @app.get("/v1/models")
    def models():
        return {"object": "list", "data": [{"id": gw.model_name, "object": "model", "owned_by": "fak-b200"}]}

    @app.get("/metrics")
    def metrics():
        from prometheus_client import generate_latest
        gw.metrics.scrape_engine(gw.backend)
        return PlainTextResponse(generate_latest(gw.metrics.registry).decode(), media_type="text/plain")

    def leased_stream(gen, body, route, priority):
        with gw.lease(body, route, priority):
            yield from gen

    def prio(req: Request) -> int | None:
        h = req.headers.get("x-fak-priority")
        return int(h) if h is not None and h.strip().lstrip("-").isdigit() else None

    @app.post("/v1/chat/completions")
    async def chat(req: Request):
        body = await req.json()
        with timed("chat"):
            if body.get("stream"):
                if gw.admission is not None and gw.admission.policy.max_waiting > 0 and \
                        gw.admission.snapshot()["waiting"] >= gw.admission.policy.max_waiting:
                    raise HTTPException(429, "server overloaded: waiting queue full")
                return StreamingResponse(leased_stream(gw.chat_completion_stream(body), body, "chat", prio(req)),
                                         media_type="text/event-stream")
            with gw.lease(body, "chat", prio(req)):
                return JSONResponse(gw.chat_completion(body))

    @app.post("/v1/completions")
    async def completions(req: Request):
        body = await req.json()
        with timed("completions"), gw.lease(body, "completions", prio(req)):
            return JSONResponse(gw.completion(body))

    @app.post("/v1/messages")
    async def messages(req: Request):
        body = await req.json()
        with timed("messages"):
            if body.get("stream"):
                return StreamingResponse(leased_stream(gw.messages_stream(body), body, "messages", prio(req)),
                                         media_type="text/event-stream")
            with gw.lease(body, "messages", prio(req)):
                return JSONResponse(gw.messages(body))

    @app.post("/v1/embeddings")
    async def embeddings(req: Request):
        body = await req.json()
        try:
            return JSONResponse(gw.embeddings(body))
        except NotImplementedError as e:
            raise HTTPException(501, str(e))

    @app.post("/v1/fak/adjudicate")
    async def adjudicate(req: Request):
        body = await req.json()
        v = gw.kernel.decide(ToolCall.from_dict(body))
        gw.metrics.verdicts.labels(v.kind.name, v.reason.name).inc()
        return v.to_dict()

    @app.get("/v1/fak/journal")
    def journal(n: int = 50):
        ok, bad = gw.kernel.journal.verify()
        return {"chain_ok": ok, "first_bad": bad, "entries": gw.kernel.journal.entries()[-n:]}

    @app.post("/v1/fak/policy")
    async def policy(req: Request):
        try:
            p = policy_from_dict(await req.json())
        except ValueError as e:
            raise HTTPException(400, str(e))
        gw.kernel.set_policy(p)
        return {"ok": True}

    from .surfaces import add_routes
    add_routes(app, gw)

    @app.get("/v1/fak/stats")
    def stats():
        out = {"kernel": dict(gw.kernel.stats)}
        eng = getattr(gw.backend, "engine", None)
        if eng is not None:
            out["engine"] = dict(eng.stats)
            if eng.radix is not None:
                out["radix"] = eng.radix.stats()
        return out

    return app
