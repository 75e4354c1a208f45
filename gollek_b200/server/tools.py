"""Tool (function) calling: prompt rendering of tool definitions and parsing of calls from output.

Formats parsed, tried in this order (the formats of the reference's parser,
runner/gguf/gollek-gguf-tokenizer/…/gguf/tokenizer/ToolCallParser.java:23-69, plus the two that
Mistral and Llama-3.1 emit):
  <tool_call>{"name": ..., "arguments": {...}}</tool_call>        Hermes / Qwen
  <function_call>{...}</function_call>
  [TOOL_CALLS] [{"name": ..., "arguments": {...}}, ...]            Mistral
  <|python_tag|>{"name": ..., "parameters": {...}}                  Llama-3.1
  Action: name  Action Input: {...}                                 ReAct
  a bare JSON object (or array of them) with "name" and "arguments" / "parameters"
JSON is cut out by a bracket scanner that respects strings, so nested objects and braces inside
string values parse (a regular expression with a lazy ``.*?`` stops at the first ``}``).
"""
from __future__ import annotations

import json
import re
import uuid
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Tuple

MARKERS = ("<tool_call>", "<function_call>", "[TOOL_CALLS]", "<|python_tag|>", "Action:")


@dataclass
class ToolCall:
    name: str
    arguments: Dict[str, Any] = field(default_factory=dict)
    id: str = field(default_factory=lambda: "call_" + uuid.uuid4().hex[:24])

    def openai(self) -> dict:
        return {"id": self.id, "type": "function",
                "function": {"name": self.name, "arguments": json.dumps(self.arguments, ensure_ascii=False)}}


def _scan_json(text: str, start: int) -> Optional[Tuple[Any, int]]:
    """Parse the JSON object or array that opens at text[start]; (value, end index) or None."""
    if start >= len(text) or text[start] not in "{[":
        return None
    depth = 0
    in_str = esc = False
    for i in range(start, len(text)):
        ch = text[i]
        if in_str:
            if esc:
                esc = False
            elif ch == "\\":
                esc = True
            elif ch == '"':
                in_str = False
        elif ch == '"':
            in_str = True
        elif ch in "{[":
            depth += 1
        elif ch in "}]":
            depth -= 1
            if depth == 0:
                try:
                    return json.loads(text[start:i + 1]), i + 1
                except json.JSONDecodeError:
                    return None
    return None


def _skip_ws(text: str, i: int) -> int:
    while i < len(text) and text[i].isspace():
        i += 1
    return i


def _as_calls(value: Any) -> List[ToolCall]:
    items = value if isinstance(value, list) else [value]
    out = []
    for it in items:
        if not isinstance(it, dict):
            continue
        if isinstance(it.get("function"), dict):  # OpenAI-shaped {"type": "function", "function": {...}}
            it = it["function"]
        name = it.get("name")
        args = it.get("arguments", it.get("parameters", {}))
        if isinstance(args, str):
            try:
                args = json.loads(args)
            except json.JSONDecodeError:
                args = {"input": args}
        if isinstance(name, str) and name.strip():
            out.append(ToolCall(name.strip(), args if isinstance(args, dict) else {"input": args}))
    return out


def _wrapped(text: str, open_tag: str, close_tag: str) -> Tuple[List[ToolCall], int]:
    calls: List[ToolCall] = []
    first = -1
    pos = 0
    while True:
        i = text.find(open_tag, pos)
        if i < 0:
            break
        first = i if first < 0 else first
        j = _skip_ws(text, i + len(open_tag))
        got = _scan_json(text, j)
        if got is None:
            pos = i + len(open_tag)
            continue
        calls.extend(_as_calls(got[0]))
        pos = got[1]
        k = _skip_ws(text, pos)
        if close_tag and text.startswith(close_tag, k):
            pos = k + len(close_tag)
    return calls, first


def _react(text: str) -> Tuple[List[ToolCall], int]:
    calls: List[ToolCall] = []
    first = -1
    for m in re.finditer(r"Action:\s*([\w.\-]+)\s*Action Input:\s*", text):
        got = _scan_json(text, m.end())
        if got is None or not isinstance(got[0], dict):
            continue
        first = m.start() if first < 0 else first
        calls.append(ToolCall(m.group(1), got[0]))
    return calls, first


def _bare(text: str) -> Tuple[List[ToolCall], int]:
    i = 0
    while i < len(text):
        j = min([k for k in (text.find("{", i), text.find("[", i)) if k >= 0], default=-1)
        if j < 0:
            break
        got = _scan_json(text, j)
        if got is not None:
            calls = _as_calls(got[0])
            if calls:
                return calls, j
            i = got[1]
        else:
            i = j + 1
    return [], -1


def parse_tool_calls(text: str) -> Tuple[str, List[ToolCall]]:
    """(content before the first call, calls); no calls -> (text, [])."""
    if not text or not text.strip():
        return text or "", []
    for open_tag, close_tag in (("<tool_call>", "</tool_call>"), ("<function_call>", "</function_call>"),
                                ("[TOOL_CALLS]", ""), ("<|python_tag|>", "")):
        calls, first = _wrapped(text, open_tag, close_tag)
        if calls:
            return text[:first].strip(), calls
    for finder in (_react, _bare):
        calls, first = finder(text)
        if calls:
            return text[:first].strip(), calls
    return text, []


def may_hold_tool_call(text: str) -> int:
    """Index from which streamed text must be held back because a tool call may be starting there
    (a marker, a prefix of one at the end, or a JSON object at the start); -1 if none."""
    best = -1
    for mk in MARKERS:
        i = text.find(mk)
        if i >= 0 and (best < 0 or i < best):
            best = i
    if best >= 0:
        return best
    s = text.lstrip()
    if s.startswith("{") or s.startswith("["):
        return len(text) - len(s)
    for mk in MARKERS:  # a marker split across stream chunks
        for k in range(len(mk) - 1, 0, -1):
            if text.endswith(mk[:k]):
                return len(text) - k
    return -1


def tools_preamble(tools: List[dict]) -> str:
    """System-prompt text that lists the tools and the call format, for chat templates without tool
    support."""
    fns = [t.get("function", t) for t in tools]
    lines = ["You can call the following functions. To call one, reply with",
             '<tool_call>{"name": <function name>, "arguments": <arguments object>}</tool_call>',
             "(one block per call) and nothing else. Functions:"]
    lines += [json.dumps(f, ensure_ascii=False) for f in fns]
    return "\n".join(lines)


def tool_choice_regex(tool_choice: Any) -> Optional[str]:
    """Output pattern for a forced tool choice: ``{"type": "function", "function": {"name": X}}``
    forces a call of X; "required" forces a call of any tool (as a bare JSON object)."""
    if isinstance(tool_choice, dict):
        name = (tool_choice.get("function") or {}).get("name")
        if name:
            return r'\{"name": "' + re.escape(name) + r'", "arguments": \{[^\n]*\}\}'
    if tool_choice == "required":
        return r'\{"name": "[A-Za-z0-9_.\-]+", "arguments": \{[^\n]*\}\}'
    return None


def messages_for_template(messages: List[dict]) -> List[dict]:
    """OpenAI tool-call history made template-friendly: assistant ``tool_calls`` arguments as objects
    and ``tool`` results kept with their call id."""
    out = []
    for m in messages:
        m = dict(m)
        if m.get("tool_calls"):
            tcs = []
            for tc in m["tool_calls"]:
                fn = dict(tc.get("function", {}))
                if isinstance(fn.get("arguments"), str):
                    try:
                        fn["arguments"] = json.loads(fn["arguments"])
                    except json.JSONDecodeError:
                        pass
                tcs.append({**tc, "function": fn})
            m["tool_calls"] = tcs
        if m.get("content") is None:
            m["content"] = ""
        out.append(m)
    return out
