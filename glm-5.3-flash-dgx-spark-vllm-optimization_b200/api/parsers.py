"""Output parsers of the OpenAI-compatible server: reasoning (``<think>`` ... ``</think>``) and tool calls.

The reference serves GLM with vLLM's ``glm45`` reasoning parser and ``glm47`` tool parser
(code/kit/launcher/start.sh:2666-2684).  This module implements the same two text conventions from their output
format, not from vLLM's code:

  reasoning   text up to the first ``</think>`` (an opening ``<think>`` is optional: the chat template may have
              emitted it) is reasoning; the rest is the answer.  Without ``</think>`` the whole text is reasoning
              while the model is still thinking, or answer text when no ``<think>`` was ever opened.
  tool calls  ``<tool_call>NAME`` followed by ``<arg_key>K</arg_key><arg_value>V</arg_value>`` pairs and
              ``</tool_call>`` (argument values that parse as JSON are kept as JSON, else as strings), or
              ``<tool_call>{"name": ..., "arguments": {...}}</tool_call>``.

``stop_index`` applies client stop strings to the answer only (stops inside the reasoning are ignored: the
reference's "suppress stops in reasoning" launcher option, REPRODUCE.md:318).
"""

from __future__ import annotations

import json
import re
import uuid

THINK_OPEN, THINK_CLOSE = "<think>", "</think>"
_TOOL_RE = re.compile(r"<tool_call>(.*?)</tool_call>", re.S)
_ARG_RE = re.compile(r"<arg_key>(.*?)</arg_key>\s*<arg_value>(.*?)</arg_value>", re.S)


def split_reasoning(text: str) -> tuple[str, str]:
    """(reasoning, answer)"""
    k = text.find(THINK_CLOSE)
    if k < 0:
        if text.lstrip().startswith(THINK_OPEN):
            return text.lstrip()[len(THINK_OPEN):], ""
        return "", text
    reasoning = text[:k]
    j = reasoning.find(THINK_OPEN)
    if j >= 0:
        reasoning = reasoning[j + len(THINK_OPEN):]
    return reasoning.strip("\n"), text[k + len(THINK_CLOSE):].lstrip("\n")


def stop_index(text: str, stops: list[str], reasoning: bool) -> int:
    """Index where the text is cut by the first stop string (-1: none).  With ``reasoning``, only matches after the
    end of the reasoning count."""
    start = 0
    if reasoning:
        k = text.find(THINK_CLOSE)
        if k < 0 and text.lstrip().startswith(THINK_OPEN):
            return -1                                   # still thinking
        start = k + len(THINK_CLOSE) if k >= 0 else 0
    best = -1
    for s in stops:
        if not s:
            continue
        k = text.find(s, start)
        if k >= 0 and (best < 0 or k < best):
            best = k
    return best


def _value(v: str):
    v = v.strip()
    try:
        return json.loads(v)
    except (ValueError, TypeError):
        return v


def parse_tool_calls(text: str) -> tuple[str, list[dict]]:
    """(content without the tool-call markup, OpenAI tool_calls)"""
    calls = []
    for m in _TOOL_RE.finditer(text):
        body = m.group(1).strip()
        name, args = None, {}
        if body.startswith("{"):
            try:
                obj = json.loads(body)
                name = obj.get("name")
                args = obj.get("arguments", obj.get("parameters", {})) or {}
                if isinstance(args, str):
                    args = _value(args)
            except ValueError:
                name = None
        else:
            first = body.split("<arg_key>", 1)[0]
            name = first.strip() or None
            args = {k.strip(): _value(v) for k, v in _ARG_RE.findall(body)}
        if name:
            calls.append({"id": f"call_{uuid.uuid4().hex[:24]}", "type": "function",
                          "function": {"name": name, "arguments": json.dumps(args, ensure_ascii=False)}})
    content = _TOOL_RE.sub("", text).strip() if calls else text
    return content, calls


def responses_input_to_messages(inp, instructions: str | None = None) -> list[dict]:
    """Responses-API ``input`` (a string or a list of items) -> chat messages.  Message items (with ``role`` and
    string or ``input_text`` / ``output_text`` content parts) are kept; items of other or unknown types
    (reasoning, function calls, images, ...) are skipped instead of being appended as malformed messages (the
    reference's responses_utils patch, code/vllm-patches/responses_utils.patch:1-17)."""
    msgs = []
    if instructions:
        msgs.append({"role": "system", "content": instructions})
    if isinstance(inp, str):
        msgs.append({"role": "user", "content": inp})
        return msgs
    for item in inp or []:
        if not isinstance(item, dict):
            continue
        typ = item.get("type", "message")
        if typ == "function_call_output":
            msgs.append({"role": "tool", "content": str(item.get("output", ""))})
            continue
        if typ != "message" or "role" not in item:
            continue
        content = item.get("content", "")
        if isinstance(content, list):
            content = "".join(p.get("text", "") for p in content
                              if isinstance(p, dict) and p.get("type", "input_text") in ("input_text", "output_text",
                                                                                         "text"))
        msgs.append({"role": item["role"], "content": content})
    return msgs
