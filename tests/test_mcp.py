"""Model Context Protocol client over stdio against a small fake MCP server: handshake, tools,
resources, prompts, errors, and the server routes that connect MCP servers and call their tools
(and offer them to the model through chat ``mcp``)."""
import os
import sys

import pytest

from gollek_b200.server.mcp import MCPClient, MCPError, MCPRegistry, tool_text

FAKE = [sys.executable, os.path.join(os.path.dirname(os.path.abspath(__file__)), "mcp_fake_server.py")]


def test_mcp_client_protocol():
    c = MCPClient(FAKE, timeout_s=20)
    try:
        info = c.initialize()
        assert info["serverInfo"]["name"] == "fake" and c.protocol_version == "2024-11-05"
        assert [t["name"] for t in c.list_tools()] == ["add", "echo"]
        assert tool_text(c.call_tool("add", {"a": 2, "b": 40})) == "42"
        assert tool_text(c.call_tool("echo", {"text": "hi"})) == "hi"
        with pytest.raises(MCPError, match="unknown tool"):
            c.call_tool("nope")
        assert c.list_resources()[0]["uri"] == "mem://readme"
        assert c.read_resource("mem://readme")["contents"][0]["text"] == "hello from the resource"
        assert c.list_prompts()[0]["name"] == "greet"
        assert "Ada" in c.get_prompt("greet", {"who": "Ada"})["messages"][0]["content"]["text"]
    finally:
        c.close()


def test_mcp_registry_openai_tools():
    r = MCPRegistry()
    try:
        r.connect("calc", FAKE)
        tools = r.openai_tools()
        assert tools[0] == {"type": "function", "function": {
            "name": "calc__add", "description": "add two integers",
            "parameters": {"type": "object", "properties": {"a": {"type": "integer"}, "b": {"type": "integer"}},
                           "required": ["a", "b"]}}}
        assert tool_text(r.call("calc__add", {"a": 1, "b": 2})) == "3"
        with pytest.raises(KeyError):
            r.call("other__add")
    finally:
        r.close()


def test_mcp_server_routes():
    from fastapi.testclient import TestClient

    from gollek_b200.config import EngineConfig, preset
    from gollek_b200.engine.engine import LLMEngine
    from gollek_b200.models.reference import init_random_weights
    from gollek_b200.server.app import create_app
    from gollek_b200.server.async_engine import AsyncEngine
    from gollek_b200.utils.tokenizer import ByteTokenizer
    cfg = preset("tiny-llama")
    w = init_random_weights(cfg, seed=0)
    ec = EngineConfig(device="cpu", dtype="float32", max_num_seqs=4, max_num_batched_tokens=256, max_model_len=1024,
                      use_cuda_graphs=False)
    eng = LLMEngine(ec, model_cfg=cfg, weights=w.__getitem__, num_blocks=96,
                    tokenizer=ByteTokenizer(cfg.vocab_size, cfg.eos_token_id))
    ae = AsyncEngine(eng).start()
    app = create_app(ae)
    try:
        with TestClient(app) as c:
            r = c.post("/v1/admin/mcp/servers", json={"name": "calc", "command": FAKE}).json()
            assert r["serverInfo"]["name"] == "fake"
            names = [t["function"]["name"] for t in c.get("/v1/mcp/tools").json()["tools"]]
            assert names == ["calc__add", "calc__echo"]
            out = c.post("/v1/mcp/tools/call", json={"name": "calc__add", "arguments": {"a": 5, "b": 6}}).json()
            assert out["text"] == "11" and out["isError"] is False
            assert c.post("/v1/mcp/tools/call", json={"name": "x__y"}).status_code == 404
            # MCP tools offered to the model: a call constrained to one of them comes back as a tool call
            call = r'\{"name": "calc__echo", "arguments": \{"text": "hi"\}\}'
            body = {"messages": [{"role": "user", "content": "echo hi"}], "mcp": True, "max_tokens": 80,
                    "guided_regex": call}
            ch = c.post("/v1/chat/completions", json=body).json()["choices"][0]
            assert ch["finish_reason"] == "tool_calls"
            assert ch["message"]["tool_calls"][0]["function"]["name"] == "calc__echo"
            assert c.delete("/v1/admin/mcp/servers/calc").status_code == 204
            assert c.get("/v1/mcp/tools").json() == {"tools": []}
    finally:
        app.state.server.mcp.close()
        ae.shutdown()
