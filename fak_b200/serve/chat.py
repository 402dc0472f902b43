"""Chat rendering (ChatML with a tools block) and tool-call extraction.

Messages in OpenAI or Anthropic shape render to ChatML turns; when tools are offered, the
system turn carries their JSON schemas and the model answers tool calls as
``<tool_call>{"name": ..., "arguments": {...}}</tool_call>`` blocks -- the convention the
Qwen2.5 / SmolLM2 instruct templates use (reference renderer: internal/agent/inkernel_render.go:40-165).
"""
from __future__ import annotations

import json
import re
import uuid
from typing import Any

TOOL_BLOCK = re.compile(r"<tool_call>\s*(\{.*?\})\s*</tool_call>", re.S)


def _content_text(content: Any) -> str:
    """OpenAI/Anthropic content (string or list of parts) -> plain text."""
    if content is None:
        return ""
    if isinstance(content, str):
        return content
    parts = []
    for p in content:
        if isinstance(p, str):
            parts.append(p)
        elif isinstance(p, dict):
            t = p.get("type")
            if t in ("text", "input_text", "output_text"):
                parts.append(p.get("text", ""))
            elif t == "tool_result":
                parts.append(f"<tool_response>\n{_content_text(p.get('content'))}\n</tool_response>")
            elif t == "tool_use":
                parts.append("<tool_call>\n" + json.dumps({"name": p.get("name"), "arguments": p.get("input", {})})
                             + "\n</tool_call>")
    return "".join(parts)


def normalize_tools(tools: list[dict] | None) -> list[dict]:
    """OpenAI ({type: function, function: {...}}) or Anthropic ({name, input_schema}) -> function specs."""
    out = []
    for t in tools or []:
        if "function" in t:
            f = t["function"]
            out.append({"name": f.get("name"), "description": f.get("description", ""),
                        "parameters": f.get("parameters", {})})
        elif "name" in t:
            out.append({"name": t["name"], "description": t.get("description", ""),
                        "parameters": t.get("input_schema", t.get("parameters", {}))})
    return out


def render_chatml(messages: list[dict], tools: list[dict] | None = None, system: str | None = None,
                  add_generation_prompt: bool = True) -> str:
    specs = normalize_tools(tools)
    sys_parts = []
    if system:
        sys_parts.append(_content_text(system))
    rest = []
    for m in messages:
        if m.get("role") == "system":
            sys_parts.append(_content_text(m.get("content")))
        else:
            rest.append(m)
    sys_text = "\n\n".join(p for p in sys_parts if p) or "You are a helpful assistant."
    if specs:
        sys_text += ("\n\n# Tools\n\nYou may call one or more functions to assist with the user query.\n\n"
                     "You are provided with function signatures within <tools></tools> XML tags:\n<tools>\n"
                     + "\n".join(json.dumps(s) for s in specs)
                     + "\n</tools>\n\nFor each function call, return a json object with function name and arguments "
                       "within <tool_call></tool_call> XML tags:\n<tool_call>\n"
                       "{\"name\": <function-name>, \"arguments\": <args-json-object>}\n</tool_call>")
    out = [f"<|im_start|>system\n{sys_text}<|im_end|>\n"]
    for m in rest:
        role = m.get("role", "user")
        text = _content_text(m.get("content"))
        if role == "assistant" and m.get("tool_calls"):
            for tc in m["tool_calls"]:
                f = tc.get("function", tc)
                args = f.get("arguments", {})
                if isinstance(args, str):
                    try:
                        args = json.loads(args)
                    except json.JSONDecodeError:
                        pass
                text += "\n<tool_call>\n" + json.dumps({"name": f.get("name"), "arguments": args}) + "\n</tool_call>"
        if role == "tool":
            role = "user"
            text = f"<tool_response>\n{text}\n</tool_response>"
        out.append(f"<|im_start|>{role}\n{text}<|im_end|>\n")
    if add_generation_prompt:
        out.append("<|im_start|>assistant\n")
    return "".join(out)


def extract_tool_calls(text: str) -> tuple[str, list[dict]]:
    """Split generated text into (plain text, [{id, name, arguments}])."""
    calls = []
    for m in TOOL_BLOCK.finditer(text):
        try:
            obj = json.loads(m.group(1))
        except json.JSONDecodeError:
            continue
        name = obj.get("name")
        if not isinstance(name, str):
            continue
        args = obj.get("arguments", obj.get("parameters", {}))
        if isinstance(args, str):
            try:
                args = json.loads(args)
            except json.JSONDecodeError:
                args = {"__raw__": args}
        calls.append({"id": "call_" + uuid.uuid4().hex[:24], "name": name, "arguments": args})
    plain = TOOL_BLOCK.sub("", text).strip()
    return plain, calls
