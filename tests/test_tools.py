"""Tool calling: parsing of the call formats, stream hold-back, templates with tools, and the
OpenAI chat API (tool_calls messages, forced calls, tool results in the history)."""
import json
import re

import pytest

from gollek_b200.config import EngineConfig, preset
from gollek_b200.engine.engine import LLMEngine
from gollek_b200.models.reference import init_random_weights
from gollek_b200.server.tools import (may_hold_tool_call, messages_for_template, parse_tool_calls,
                                      tool_choice_regex, tools_preamble)
from gollek_b200.utils.tokenizer import ByteTokenizer, default_chat_template

WEATHER = {"type": "function", "function": {"name": "get_weather", "description": "weather by city",
                                            "parameters": {"type": "object",
                                                           "properties": {"city": {"type": "string"}}}}}


@pytest.mark.parametrize("text,name,args,before", [
    ('<tool_call>{"name": "get_weather", "arguments": {"city": "Paris"}}</tool_call>', "get_weather",
     {"city": "Paris"}, ""),
    ('Let me check.\n<tool_call>\n{"name": "f", "arguments": {"q": {"deep": [1, {"x": "}"}]}}}\n</tool_call>', "f",
     {"q": {"deep": [1, {"x": "}"}]}}, "Let me check."),
    ('<function_call>{"name": "g", "parameters": {"a": 1}}</function_call>', "g", {"a": 1}, ""),
    ('[TOOL_CALLS] [{"name": "h", "arguments": {"b": true}}]', "h", {"b": True}, ""),
    ('<|python_tag|>{"name": "k", "parameters": {"n": 3}}', "k", {"n": 3}, ""),
    ('Thought: need data\nAction: search\nAction Input: {"query": "b200"}', "search", {"query": "b200"},
     "Thought: need data"),
    ('{"name": "m", "arguments": "{\\"s\\": 2}"}', "m", {"s": 2}, ""),
    ('{"type": "function", "function": {"name": "n", "arguments": {}}}', "n", {}, ""),
])
def test_parse_formats(text, name, args, before):
    content, calls = parse_tool_calls(text)
    assert len(calls) == 1
    assert calls[0].name == name and calls[0].arguments == args
    assert content == before
    oa = calls[0].openai()
    assert oa["type"] == "function" and json.loads(oa["function"]["arguments"]) == args
    assert oa["id"].startswith("call_")


def test_parse_multiple_and_none():
    text = ('<tool_call>{"name": "a", "arguments": {}}</tool_call>'
            '<tool_call>{"name": "b", "arguments": {"x": 1}}</tool_call>')
    _, calls = parse_tool_calls(text)
    assert [c.name for c in calls] == ["a", "b"]
    _, calls = parse_tool_calls('[TOOL_CALLS] [{"name": "a", "arguments": {}}, {"name": "b", "arguments": {}}]')
    assert [c.name for c in calls] == ["a", "b"]
    for plain in ("The weather is nice.", '{"city": "Paris"}', "<tool_call>{not json}</tool_call>", ""):
        content, calls = parse_tool_calls(plain)
        assert calls == [] and content == plain


def test_stream_hold_back():
    assert may_hold_tool_call("Sure, checking") == -1
    assert may_hold_tool_call("Sure <tool_call>{") == 5
    assert may_hold_tool_call("Sure <tool_") == 5       # a marker split across chunks
    assert may_hold_tool_call('  {"name"') == 2
    assert may_hold_tool_call("x [TOOL_CALLS]") == 2


def test_tool_choice_regex_matches_calls():
    rx = tool_choice_regex({"type": "function", "function": {"name": "get_weather"}})
    assert re.fullmatch(rx, '{"name": "get_weather", "arguments": {"city": "Rome"}}')
    assert not re.fullmatch(rx, '{"name": "other", "arguments": {}}')
    assert re.fullmatch(tool_choice_regex("required"), '{"name": "x_1", "arguments": {}}')
    assert tool_choice_regex("auto") is None


def test_templates_with_tools():
    msgs = [{"role": "user", "content": "weather in Paris?"}]
    p = default_chat_template(msgs, [WEATHER])
    assert "get_weather" in p and "<tool_call>" in p and p.endswith("<|assistant|>\n")
    assert "get_weather" in tools_preamble([WEATHER])
    hist = messages_for_template(msgs + [
        {"role": "assistant", "content": None,
         "tool_calls": [{"id": "call_1", "type": "function",
                         "function": {"name": "get_weather", "arguments": '{"city": "Paris"}'}}]},
        {"role": "tool", "tool_call_id": "call_1", "content": "18C"}])
    assert hist[1]["tool_calls"][0]["function"]["arguments"] == {"city": "Paris"}
    p = default_chat_template(hist)
    assert '"city": "Paris"' in p and "18C" in p


def _engine():
    cfg = preset("tiny-llama")
    w = init_random_weights(cfg, seed=0)
    ec = EngineConfig(device="cpu", dtype="float32", max_num_seqs=4, max_num_batched_tokens=64, max_model_len=512,
                      use_cuda_graphs=False)
    return LLMEngine(ec, model_cfg=cfg, weights=w.__getitem__, num_blocks=96,
                     tokenizer=ByteTokenizer(cfg.vocab_size, cfg.eos_token_id))


def test_api_tool_calls():
    from fastapi.testclient import TestClient

    from gollek_b200.server.app import create_app
    from gollek_b200.server.async_engine import AsyncEngine
    call = r'\{"name": "get_weather", "arguments": \{"city": "Oslo"\}\}'
    ae = AsyncEngine(_engine()).start()
    try:
        with TestClient(create_app(ae)) as c:
            body = {"messages": [{"role": "user", "content": "weather?"}], "tools": [WEATHER], "max_tokens": 80,
                    "guided_regex": call}
            j = c.post("/v1/chat/completions", json=body).json()
            ch = j["choices"][0]
            assert ch["finish_reason"] == "tool_calls", j
            tc = ch["message"]["tool_calls"][0]
            assert tc["function"]["name"] == "get_weather"
            assert json.loads(tc["function"]["arguments"]) == {"city": "Oslo"}
            assert ch["message"]["content"] is None
            # streamed: no text deltas of the call, one tool_calls delta, finish_reason tool_calls
            with c.stream("POST", "/v1/chat/completions", json={**body, "stream": True}) as r:
                lines = [ln for ln in r.iter_lines() if ln.startswith("data: ")]
            assert lines[-1] == "data: [DONE]"
            chunks = [json.loads(ln[6:]) for ln in lines[:-1]]
            deltas = [ch["choices"][0]["delta"] for ch in chunks if ch["choices"]]
            assert all("get_weather" not in (d.get("content") or "") for d in deltas)
            tcs = [d["tool_calls"] for d in deltas if "tool_calls" in d]
            assert len(tcs) == 1 and tcs[0][0]["function"]["name"] == "get_weather"
            assert any(ch["choices"] and ch["choices"][0]["finish_reason"] == "tool_calls" for ch in chunks)
            # tool results in the history, tool_choice none: plain text answer
            hist = body["messages"] + [{"role": "assistant", "content": None, "tool_calls": [tc]},
                                       {"role": "tool", "tool_call_id": tc["id"], "content": "-3C"}]
            j = c.post("/v1/chat/completions", json={"messages": hist, "tools": [WEATHER], "tool_choice": "none",
                                                     "max_tokens": 5, "guided_regex": "cold"}).json()
            assert j["choices"][0]["message"]["content"] == "cold"
            assert "tool_calls" not in j["choices"][0]["message"]
    finally:
        ae.shutdown(drain=False)
