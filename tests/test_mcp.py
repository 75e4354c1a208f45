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


# ------------------------------------------------------------------------------ HTTP transports
def _http_server():
    """A fake MCP server speaking both HTTP transports: streamable HTTP at /mcp (JSON replies, an
    event-stream reply for tools/call, a session id required after initialize) and HTTP+SSE at
    /sse (endpoint event) + /messages."""
    import json as _json
    import queue as _queue
    import threading
    from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
    from tests.mcp_fake_server import handle

    sessions: dict = {}  # SSE session id -> queue of that connection's outgoing messages
    sse_q: "_queue.Queue" = _queue.Queue()  # closes every SSE stream when None is put

    class H(BaseHTTPRequestHandler):
        def log_message(self, *a):
            pass

        def _body(self):
            return _json.loads(self.rfile.read(int(self.headers.get("Content-Length", 0))))

        def do_POST(self):
            if self.path.startswith("/messages"):
                sid = self.path.split("session=")[-1]
                rep = handle(self._body())
                if rep is not None and sid in sessions:
                    sessions[sid].put(rep)
                self.send_response(202)
                self.end_headers()
                return
            req = self._body()
            if req.get("method") != "initialize" and self.headers.get("Mcp-Session-Id") != "s-1":
                self.send_response(400)
                self.end_headers()
                return
            rep = handle(req)
            if rep is None:
                self.send_response(202)
                self.end_headers()
                return
            if req.get("method") == "tools/call":  # reply as an event stream
                body = ("event: message\ndata: " + _json.dumps(rep) + "\n\n").encode()
                self.send_response(200)
                self.send_header("Content-Type", "text/event-stream")
            else:
                body = _json.dumps(rep).encode()
                self.send_response(200)
                self.send_header("Content-Type", "application/json")
            if req.get("method") == "initialize":
                self.send_header("Mcp-Session-Id", "s-1")
            self.send_header("Content-Length", str(len(body)))
            self.end_headers()
            self.wfile.write(body)

        def do_GET(self):
            if self.path != "/sse":
                self.send_response(404)
                self.end_headers()
                return
            sid = str(len(sessions) + 1)
            mine: "_queue.Queue" = _queue.Queue()
            sessions[sid] = mine
            self.send_response(200)
            self.send_header("Content-Type", "text/event-stream")
            self.end_headers()
            self.wfile.write(f"event: endpoint\ndata: /messages?session={sid}\n\n".encode())
            self.wfile.flush()
            while True:
                try:
                    rep = mine.get(timeout=0.2)
                except _queue.Empty:
                    if not sse_q.empty():
                        return
                    continue
                if rep is None:
                    return
                try:
                    self.wfile.write(("event: message\ndata: " + _json.dumps(rep) + "\n\n").encode())
                    self.wfile.flush()
                except OSError:
                    return

        def do_DELETE(self):
            self.send_response(200)
            self.end_headers()

    srv = ThreadingHTTPServer(("127.0.0.1", 0), H)
    srv.daemon_threads = True
    threading.Thread(target=srv.serve_forever, daemon=True).start()
    return srv, sse_q


@pytest.mark.parametrize("transport,path", [("http", "/mcp"), ("sse", "/sse")])
def test_mcp_http_transports(transport, path):
    srv, q = _http_server()
    url = f"http://127.0.0.1:{srv.server_address[1]}{path}"
    c = MCPClient(url=url, transport=transport, timeout_s=10)
    try:
        info = c.initialize()
        assert info["serverInfo"]["name"] == "fake"
        if transport == "http":
            assert c.session_id == "s-1"
        assert [t["name"] for t in c.list_tools()] == ["add", "echo"]
        assert tool_text(c.call_tool("add", {"a": 20, "b": 22})) == "42"
        with pytest.raises(MCPError, match="unknown tool"):
            c.call_tool("nope")
        r = MCPRegistry()
        r.connect("web", url=url, transport=transport, timeout_s=10)
        assert tool_text(r.call("web__echo", {"text": "over http"})) == "over http"
        r.close()
    finally:
        c.close()
        q.put(None)
        q.put(None)
        srv.shutdown()
