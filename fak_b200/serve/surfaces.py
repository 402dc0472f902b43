"""The gateway's other wire surfaces, all routed through the same adjudicated generation path.

  POST /v1/responses                  OpenAI Responses API (buffered; ``stream: true`` is refused)
  POST /v1/messages/count_tokens      Anthropic token count of a messages request (exact tokenizer count)
  POST /v1/moderations                OpenAI moderations wire with a deterministic lexical classifier
  POST /v1beta/models/{m}:generateContent, :countTokens   Gemini wire
  POST /v1/fak/syscall                adjudicate + execute one tool call through the kernel
  POST /v1/fak/admit                  run a client-produced tool result through the context MMU
  POST /mcp                           MCP over HTTP (JSON-RPC 2.0: initialize, ping, tools/list, tools/call)
  GET  /a2a/v1/agent-card, POST /a2a/v1/messages, GET /a2a/v1/tasks[/{id}], POST /a2a/v1/tasks/{id}/cancel
  GET  /v1/fak/admission, GET /v1/fak/autoscale   admission-controller and autoscaler views

Every surface that generates converts its request into the chat form, calls
``Gateway.chat_completion`` -- so proposed tool calls are adjudicated by the kernel on every path --
and converts the answer back.  Reference surface: internal/gateway/http.go:54-131 (responses.go,
messages.go:1361 count_tokens, moderations.go, gemini.go, http.go:994-1050 syscall / admit, mcp.go,
a2a.go); the handlers here are this package's own.
"""
from __future__ import annotations

import json
import threading
import time
import uuid
from typing import Any

from fastapi import FastAPI, HTTPException, Request
from fastapi.responses import JSONResponse, Response

from ..agentkernel import ToolCall

# ---------------------------------------------------------------------------- conversions


def _text_of(content) -> str:
    """Text of a content field: a string, or a list of typed parts (input_text / output_text / text)."""
    if content is None:
        return ""
    if isinstance(content, str):
        return content
    out = []
    for p in content:
        if isinstance(p, str):
            out.append(p)
        elif isinstance(p, dict) and isinstance(p.get("text"), str):
            out.append(p["text"])
    return "".join(out)


def responses_to_chat(body: dict) -> dict:
    """OpenAI Responses request -> chat-completions request."""
    if body.get("stream"):
        raise HTTPException(400, "stream: true is not supported on /v1/responses (buffered only)")
    msgs: list[dict] = []
    if body.get("instructions"):
        msgs.append({"role": "system", "content": str(body["instructions"])})
    inp = body.get("input", "")
    if isinstance(inp, str):
        msgs.append({"role": "user", "content": inp})
    else:
        for item in inp:
            t = item.get("type", "message")
            if t == "message" or "role" in item and t not in ("function_call", "function_call_output"):
                role = item.get("role", "user")
                msgs.append({"role": "system" if role == "developer" else role, "content": _text_of(item.get("content"))})
            elif t == "function_call":
                args = item.get("arguments") or "{}"
                msgs.append({"role": "assistant", "content": None,
                             "tool_calls": [{"id": item.get("call_id", ""), "type": "function",
                                             "function": {"name": item.get("name", ""), "arguments": args}}]})
            elif t == "function_call_output":
                msgs.append({"role": "tool", "tool_call_id": item.get("call_id", ""),
                             "content": _text_of(item.get("output"))})
            else:
                raise HTTPException(400, f"unsupported input item type {t!r}")
    tools = []
    for t in body.get("tools") or []:
        if t.get("type") == "function":
            tools.append({"type": "function", "function": {k: t[k] for k in ("name", "description", "parameters")
                                                           if k in t}})
    out = {"messages": msgs, "max_tokens": body.get("max_output_tokens"), "tools": tools or None}
    for k in ("temperature", "top_p", "seed"):
        if k in body:
            out[k] = body[k]
    return out


def chat_to_responses(resp: dict, model: str) -> dict:
    msg = resp["choices"][0]["message"]
    output: list[dict] = []
    if msg.get("content"):
        output.append({"type": "message", "id": "msg_" + uuid.uuid4().hex[:24], "role": "assistant",
                       "status": "completed",
                       "content": [{"type": "output_text", "text": msg["content"], "annotations": []}]})
    for tc in msg.get("tool_calls") or []:
        output.append({"type": "function_call", "id": "fc_" + uuid.uuid4().hex[:24], "call_id": tc["id"],
                       "name": tc["function"]["name"], "arguments": tc["function"]["arguments"],
                       "status": "completed"})
    u = resp.get("usage", {})
    inc = resp["choices"][0].get("finish_reason") == "length"
    return {"id": "resp_" + uuid.uuid4().hex[:24], "object": "response", "created_at": int(time.time()),
            "model": model, "status": "incomplete" if inc else "completed",
            "incomplete_details": {"reason": "max_output_tokens"} if inc else None, "output": output,
            "usage": {"input_tokens": u.get("prompt_tokens", 0), "output_tokens": u.get("completion_tokens", 0),
                      "total_tokens": u.get("prompt_tokens", 0) + u.get("completion_tokens", 0)}}


def gemini_to_chat(body: dict) -> dict:
    msgs: list[dict] = []
    si = body.get("systemInstruction") or body.get("system_instruction")
    if si:
        msgs.append({"role": "system", "content": _text_of(si.get("parts", []))})
    for c in body.get("contents", []):
        role = "assistant" if c.get("role") == "model" else "user"
        text, calls, results = [], [], []
        for p in c.get("parts", []):
            if "text" in p:
                text.append(p["text"])
            elif "functionCall" in p:
                fc = p["functionCall"]
                calls.append({"id": "call_" + uuid.uuid4().hex[:12], "type": "function",
                              "function": {"name": fc.get("name", ""), "arguments": json.dumps(fc.get("args", {}))}})
            elif "functionResponse" in p:
                fr = p["functionResponse"]
                results.append({"role": "tool", "tool_call_id": fr.get("name", ""),
                                "content": json.dumps(fr.get("response", {}))})
        if text or calls:
            m: dict[str, Any] = {"role": role, "content": "".join(text) or None}
            if calls:
                m["tool_calls"] = calls
            msgs.append(m)
        msgs.extend(results)
    tools = []
    for t in body.get("tools") or []:
        for fd in t.get("functionDeclarations") or t.get("function_declarations") or []:
            tools.append({"type": "function", "function": {k: fd[k] for k in ("name", "description", "parameters")
                                                           if k in fd}})
    gc = body.get("generationConfig") or {}
    out = {"messages": msgs, "tools": tools or None, "max_tokens": gc.get("maxOutputTokens")}
    for src, dst in (("temperature", "temperature"), ("topP", "top_p"), ("topK", "top_k")):
        if src in gc:
            out[dst] = gc[src]
    if gc.get("stopSequences"):
        out["stop"] = gc["stopSequences"]
    return out


def chat_to_gemini(resp: dict, model: str) -> dict:
    ch = resp["choices"][0]
    msg = ch["message"]
    parts: list[dict] = []
    if msg.get("content"):
        parts.append({"text": msg["content"]})
    for tc in msg.get("tool_calls") or []:
        parts.append({"functionCall": {"name": tc["function"]["name"],
                                       "args": json.loads(tc["function"]["arguments"] or "{}")}})
    u = resp.get("usage", {})
    return {"candidates": [{"content": {"role": "model", "parts": parts}, "index": 0,
                            "finishReason": "MAX_TOKENS" if ch.get("finish_reason") == "length" else "STOP"}],
            "usageMetadata": {"promptTokenCount": u.get("prompt_tokens", 0),
                              "candidatesTokenCount": u.get("completion_tokens", 0),
                              "totalTokenCount": u.get("prompt_tokens", 0) + u.get("completion_tokens", 0)},
            "modelVersion": model}


# ---------------------------------------------------------------------------- moderation
# The public OpenAI category keys; each scored by a small lexicon of this package's choosing.
MODERATION_LEXICON: dict[str, tuple[str, ...]] = {
    "harassment": ("idiot", "loser", "pathetic", "worthless", "stupid"),
    "harassment/threatening": ("i will hurt you", "watch your back", "you will regret", "i'll find you"),
    "hate": ("subhuman", "vermin", "inferior race", "go back to your country"),
    "hate/threatening": ("exterminate them", "wipe them out"),
    "illicit": ("buy drugs", "launder money", "counterfeit", "stolen credit card", "pick a lock"),
    "illicit/violent": ("build a bomb", "make a weapon", "untraceable gun"),
    "self-harm": ("hurt myself", "self harm", "self-harm", "end my life"),
    "self-harm/intent": ("i want to die", "kill myself", "end it all"),
    "self-harm/instructions": ("how to overdose", "ways to cut myself"),
    "sexual": ("explicit sex", "nude", "porn"),
    "sexual/minors": ("underage sex", "child porn"),
    "violence": ("kill", "murder", "stab", "shoot", "beat up"),
    "violence/graphic": ("gore", "dismember", "blood everywhere"),
}
MODERATION_THRESHOLD = 0.5


def moderate(text: str) -> dict:
    """Score = 1 - 0.6 ** hits per category (one hit 0.4, two 0.64); flagged at >= 0.5."""
    hay = text.lower()
    scores, cats = {}, {}
    for cat, words in MODERATION_LEXICON.items():
        hits = sum(hay.count(w) for w in words)
        s = round(1.0 - 0.6 ** hits, 4) if hits else 0.0
        scores[cat] = s
        cats[cat] = s >= MODERATION_THRESHOLD
    return {"flagged": any(cats.values()), "categories": cats, "category_scores": scores}


# ---------------------------------------------------------------------------- A2A tasks
class TaskStore:
    """A2A tasks of this gateway (in memory, newest last)."""

    def __init__(self, cap: int = 1024):
        self.tasks: dict[str, dict] = {}
        self.cap = cap
        self._lock = threading.Lock()

    def put(self, t: dict) -> None:
        with self._lock:
            self.tasks[t["id"]] = t
            while len(self.tasks) > self.cap:
                self.tasks.pop(next(iter(self.tasks)))

    def get(self, tid: str) -> dict | None:
        with self._lock:
            return self.tasks.get(tid)

    def list(self) -> list[dict]:
        with self._lock:
            return list(self.tasks.values())


def agent_card(gw) -> dict:
    tools = sorted(gw.kernel.handlers)
    return {"name": gw.model_name, "description": "fak-b200 gateway: an LLM behind a default-deny tool-call floor",
            "url": "/a2a/v1", "version": "1", "protocolVersion": "0.3",
            "capabilities": {"streaming": False, "pushNotifications": False},
            "defaultInputModes": ["text/plain"], "defaultOutputModes": ["text/plain"],
            "skills": [{"id": "chat", "name": "chat", "description": "adjudicated chat completion"}]
            + [{"id": t, "name": t, "description": "kernel tool"} for t in tools]}


# ---------------------------------------------------------------------------- routes
def add_routes(app: FastAPI, gw) -> None:
    tasks = TaskStore()

    def generate(chat_body: dict, route: str) -> dict:
        with gw.lease(chat_body, route):
            return gw.chat_completion(chat_body)

    @app.post("/v1/responses")
    async def responses(req: Request):
        body = await req.json()
        chat_body = responses_to_chat(body)
        return JSONResponse(chat_to_responses(generate(chat_body, "responses"), body.get("model") or gw.model_name))

    @app.post("/v1/messages/count_tokens")
    async def count_tokens(req: Request):
        body = await req.json()
        if not isinstance(body.get("messages"), list):
            raise HTTPException(400, "malformed request body: messages must be a list")
        return {"input_tokens": gw.count_prompt_tokens(gw._anthropic_prompt(body))}

    @app.post("/v1/moderations")
    async def moderations(req: Request):
        body = await req.json()
        inp = body.get("input", "")
        items = [inp] if isinstance(inp, str) else list(inp)
        if not all(isinstance(x, str) for x in items):
            raise HTTPException(400, "input must be a string or a list of strings")
        return {"id": "modr-" + uuid.uuid4().hex[:24], "model": body.get("model") or "fak-lexical-moderation",
                "results": [moderate(x) for x in items]}

    @app.post("/v1beta/models/{target}")
    async def gemini(target: str, req: Request):
        body = await req.json()
        model, _, method = target.partition(":")
        chat_body = gemini_to_chat(body)
        if method == "countTokens":
            from .chat import render_chatml
            return {"totalTokens": gw.count_prompt_tokens(render_chatml(chat_body["messages"], chat_body.get("tools")))}
        if method != "generateContent":
            raise HTTPException(404, f"unsupported Gemini method {method!r}")
        return JSONResponse(chat_to_gemini(generate(chat_body, "gemini"), model or gw.model_name))

    @app.post("/v1/fak/syscall")
    async def syscall(req: Request):
        body = await req.json()
        call = ToolCall.from_dict(body)
        res = gw.kernel.syscall(call)
        gw.metrics.verdicts.labels(res.verdict.kind.name, res.verdict.reason.name).inc()
        return {"verdict": res.verdict.to_dict(), "status": res.status.name,
                "result": res.payload if isinstance(res.payload, (str, int, float, bool, type(None), list, dict))
                else str(res.payload), "trace_id": call.trace_id}

    @app.post("/v1/fak/admit")
    async def admit(req: Request):
        body = await req.json()
        tool = body.get("tool") or body.get("name")
        if not tool:
            raise HTTPException(400, "admit: tool is required")
        result = body.get("result", "")
        content = result if isinstance(result, str) else json.dumps(result)
        adm = gw.kernel.mmu.admit(str(tool), content)
        gw.kernel.journal.append("admission", tool=str(tool), verdict=adm.verdict.to_dict(),
                                 findings=len(adm.findings), trace_id=body.get("trace_id", ""))
        return {"verdict": adm.verdict.to_dict(), "result": adm.content, "findings": len(adm.findings),
                "trace_id": body.get("trace_id", "")}

    @app.post("/mcp")
    async def mcp(req: Request):
        msg = await req.json()
        if isinstance(msg, list):
            out = [r for r in (mcp_dispatch(gw, m) for m in msg) if r is not None]
            return JSONResponse(out) if out else Response(status_code=202)
        r = mcp_dispatch(gw, msg)
        return JSONResponse(r) if r is not None else Response(status_code=202)

    @app.get("/a2a/v1/agent-card")
    def a2a_card():
        return agent_card(gw)

    @app.post("/a2a/v1/messages")
    async def a2a_send(req: Request):
        body = await req.json()
        m = body.get("message") or body
        text = "".join(p.get("text", "") for p in m.get("parts", []) if isinstance(p, dict))
        tid = "task-" + uuid.uuid4().hex[:16]
        task = {"id": tid, "contextId": m.get("contextId") or tid, "kind": "task",
                "status": {"state": "working", "timestamp": time.time()}, "history": [m], "artifacts": []}
        tasks.put(task)
        try:
            resp = generate({"messages": [{"role": "user", "content": text}],
                             "max_tokens": body.get("max_tokens")}, "a2a")
            reply = resp["choices"][0]["message"].get("content") or ""
            task["artifacts"].append({"artifactId": "art-" + uuid.uuid4().hex[:12],
                                      "parts": [{"kind": "text", "text": reply}]})
            task["history"].append({"role": "agent", "parts": [{"kind": "text", "text": reply}]})
            task["status"] = {"state": "completed", "timestamp": time.time()}
        except HTTPException:
            task["status"] = {"state": "rejected", "timestamp": time.time()}
            raise
        return task

    @app.get("/a2a/v1/tasks")
    def a2a_tasks():
        return {"tasks": tasks.list()}

    @app.get("/a2a/v1/tasks/{tid}")
    def a2a_task(tid: str):
        t = tasks.get(tid)
        if t is None:
            raise HTTPException(404, "no such task")
        return t

    @app.post("/a2a/v1/tasks/{tid}/cancel")
    def a2a_cancel(tid: str):
        t = tasks.get(tid)
        if t is None:
            raise HTTPException(404, "no such task")
        if t["status"]["state"] in ("completed", "failed", "rejected", "canceled"):
            raise HTTPException(409, f"task already {t['status']['state']}")
        t["status"] = {"state": "canceled", "timestamp": time.time()}
        return t

    @app.get("/v1/fak/admission")
    def admission():
        return gw.admission.snapshot() if gw.admission is not None else {"enabled": False}

    @app.get("/v1/fak/autoscale")
    def autoscale(replicas: int = 1):
        return gw.autoscale_decision(replicas)


MCP_PROTOCOL = "2025-03-26"


def mcp_dispatch(gw, msg: dict) -> dict | None:
    """One JSON-RPC 2.0 message; None for notifications (no id)."""
    mid = msg.get("id")
    method = msg.get("method", "")
    params = msg.get("params") or {}

    def ok(result):
        return {"jsonrpc": "2.0", "id": mid, "result": result}

    def err(code, text):
        return {"jsonrpc": "2.0", "id": mid, "error": {"code": code, "message": text}}

    if mid is None:
        return None   # notifications (notifications/initialized, cancelled) need no answer
    if method == "initialize":
        return ok({"protocolVersion": MCP_PROTOCOL, "capabilities": {"tools": {"listChanged": False}},
                   "serverInfo": {"name": "fak-b200", "version": "1"}})
    if method == "ping":
        return ok({})
    if method == "tools/list":
        schemas = getattr(gw.kernel.preflight, "schemas", {}) or {}
        return ok({"tools": [{"name": t, "description": f"kernel tool {t}",
                              "inputSchema": schemas.get(t) or {"type": "object"}}
                             for t in sorted(gw.kernel.handlers)]})
    if method == "tools/call":
        name = params.get("name")
        if not name:
            return err(-32602, "tools/call: name is required")
        call = ToolCall(tool=str(name), args=params.get("arguments") or {}, trace_id=str(mid))
        res = gw.kernel.syscall(call)
        gw.metrics.verdicts.labels(res.verdict.kind.name, res.verdict.reason.name).inc()
        if res.status.name != "OK":
            text = f"refused: {res.verdict.reason.name}" if not res.verdict.allowed else str(res.payload)
            return ok({"content": [{"type": "text", "text": text}], "isError": True})
        out = res.payload if isinstance(res.payload, str) else json.dumps(res.payload)
        return ok({"content": [{"type": "text", "text": out}], "isError": False})
    return err(-32601, f"method not found: {method}")
