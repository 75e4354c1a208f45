"""Model Context Protocol client (stdio, HTTP+SSE and streamable HTTP transports) and registry of
connected MCP servers.

Reference behaviour: plugins/gollek-plugin-mcp/…/mcp/dto/MCPConnection.java:82-170 (``initialize``
with the client's protocol version and capabilities, then ``notifications/initialized``,
``tools/list``), MCPToolExecutor / MCPResourceProvider / MCPPromptProvider (``tools/call``,
``resources/list`` + ``resources/read``, ``prompts/list`` + ``prompts/get``) and StdioTransport
(the server runs as a child process; JSON-RPC 2.0 messages, one per line, on its stdin / stdout),
and the protocol's HTTP transports (plugins/gollek-plugin-mcp/…/mcp/protocol/McpProtocol.java):
``sse`` — a GET opens a server-sent-event stream whose first ``endpoint`` event names the URL the
client POSTs its messages to, replies arrive as ``message`` events; ``http`` (streamable HTTP) —
every message is a POST whose response is the reply as JSON or as an event stream, with the
``Mcp-Session-Id`` the server assigned at initialisation sent back on every later POST.
MCP tools are offered to the model as OpenAI function tools (``openai_tools``), so the server's
tool calling and constrained decoding work with them unchanged.
"""
from __future__ import annotations

import json
import queue
import subprocess
import threading
from typing import Any, Dict, List, Optional

PROTOCOL_VERSION = "2024-11-05"


class MCPError(RuntimeError):
    pass


def _sse_events(lines):
    """(event, data) pairs of a server-sent-event stream given as an iterator of text lines."""
    event, data = "message", []
    for raw in lines:
        line = raw.decode("utf-8") if isinstance(raw, bytes) else raw
        line = line.rstrip("\r\n")
        if not line:
            if data:
                yield event, "\n".join(data)
            event, data = "message", []
            continue
        if line.startswith(":"):
            continue
        key, _, val = line.partition(":")
        val = val[1:] if val.startswith(" ") else val
        if key == "event":
            event = val
        elif key == "data":
            data.append(val)
    if data:
        yield event, "\n".join(data)


class MCPClient:
    """One MCP server connection. ``command`` runs a stdio server; ``url`` with ``transport``
    "sse" or "http" connects to an HTTP server."""

    def __init__(self, command: Optional[List[str]] = None, timeout_s: float = 30.0, env: Optional[dict] = None,
                 url: Optional[str] = None, transport: str = "stdio", headers: Optional[dict] = None):
        self.timeout_s = timeout_s
        self._q: "queue.Queue[dict]" = queue.Queue()
        self._next_id = 1
        self._lock = threading.Lock()
        self.server_info: dict = {}
        self.protocol_version: Optional[str] = None
        self.transport = transport if url else "stdio"
        self.url = url
        self.headers = dict(headers or {})
        self.proc = None
        self.session_id: Optional[str] = None
        self._closed = False
        if self.transport == "stdio":
            if not command:
                raise ValueError("a stdio MCP server needs a command")
            self.proc = subprocess.Popen(command, stdin=subprocess.PIPE, stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True, bufsize=1, env=env)
            threading.Thread(target=self._reader, daemon=True).start()
        elif self.transport == "sse":
            import requests
            self._http = requests.Session()
            self._post_url: Optional[str] = None
            self._endpoint = threading.Event()
            self._sse = self._http.get(url, headers={**self.headers, "Accept": "text/event-stream"}, stream=True,
                                       timeout=(timeout_s, None))
            self._sse.raise_for_status()
            threading.Thread(target=self._sse_reader, daemon=True).start()
            if not self._endpoint.wait(timeout_s):
                raise MCPError("MCP SSE server sent no endpoint event")
        elif self.transport == "http":
            import requests
            self._http = requests.Session()
        else:
            raise ValueError(f"unknown MCP transport {transport!r} (stdio, sse, http)")

    # -- stdio
    def _reader(self) -> None:
        for line in self.proc.stdout:
            line = line.strip()
            if not line:
                continue
            try:
                self._q.put(json.loads(line))
            except json.JSONDecodeError:
                continue  # a server's stray log line
        self._q.put({"_eof": True})

    # -- HTTP + SSE
    def _sse_reader(self) -> None:
        from urllib.parse import urljoin
        def lines():  # line by line as they arrive (iter_lines would wait for a full chunk)
            while True:
                line = self._sse.raw.readline()
                if not line:
                    return
                yield line

        try:
            for event, data in _sse_events(lines()):
                if event == "endpoint":
                    self._post_url = urljoin(self.url, data.strip())
                    self._endpoint.set()
                elif event == "message":
                    self._queue_json(data)
        except Exception:
            pass
        self._q.put({"_eof": True})

    def _queue_json(self, text: str) -> None:
        try:
            msg = json.loads(text)
        except json.JSONDecodeError:
            return
        for m in (msg if isinstance(msg, list) else [msg]):
            self._q.put(m)

    def _send(self, msg: dict) -> None:
        if self.transport == "stdio":
            if self.proc.poll() is not None:
                raise MCPError("MCP server exited")
            self.proc.stdin.write(json.dumps(msg) + "\n")
            self.proc.stdin.flush()
            return
        if self.transport == "sse":
            r = self._http.post(self._post_url, json=msg, headers=self.headers, timeout=self.timeout_s)
            if r.status_code >= 400:
                raise MCPError(f"MCP POST failed: HTTP {r.status_code}")
            return
        hdrs = {**self.headers, "Accept": "application/json, text/event-stream", "Content-Type": "application/json"}
        if self.session_id:
            hdrs["Mcp-Session-Id"] = self.session_id
        r = self._http.post(self.url, json=msg, headers=hdrs, timeout=self.timeout_s, stream=True)
        if r.status_code >= 400:
            raise MCPError(f"MCP POST failed: HTTP {r.status_code}")
        sid = r.headers.get("Mcp-Session-Id")
        if sid:
            self.session_id = sid
        ctype = r.headers.get("Content-Type", "")
        if "text/event-stream" in ctype:
            for event, data in _sse_events(r.iter_lines(decode_unicode=True)):
                if event == "message":
                    self._queue_json(data)
        elif r.content:
            self._queue_json(r.text)

    def request(self, method: str, params: Optional[dict] = None) -> Any:
        """One JSON-RPC request; returns its ``result`` (raises MCPError on an error reply or timeout).
        Notifications and replies to other ids that arrive meanwhile are skipped."""
        with self._lock:
            rid = self._next_id
            self._next_id += 1
            self._send({"jsonrpc": "2.0", "id": rid, "method": method, **({"params": params} if params else {})})
            while True:
                try:
                    msg = self._q.get(timeout=self.timeout_s)
                except queue.Empty:
                    raise MCPError(f"{method}: no reply within {self.timeout_s:g} s")
                if msg.get("_eof"):
                    raise MCPError(f"{method}: MCP server closed the connection")
                if msg.get("id") != rid:
                    continue
                if "error" in msg:
                    e = msg["error"]
                    raise MCPError(f"{method}: {e.get('message', e)} (code {e.get('code')})")
                return msg.get("result")

    def notify(self, method: str, params: Optional[dict] = None) -> None:
        with self._lock:
            self._send({"jsonrpc": "2.0", "method": method, **({"params": params} if params else {})})

    def initialize(self, client_name: str = "gollek-b200", version: str = "0.1") -> dict:
        res = self.request("initialize", {"protocolVersion": PROTOCOL_VERSION, "capabilities": {},
                                          "clientInfo": {"name": client_name, "version": version}})
        self.protocol_version = (res or {}).get("protocolVersion")
        self.server_info = (res or {}).get("serverInfo", {})
        self.notify("notifications/initialized")
        return res

    def list_tools(self) -> List[dict]:
        return (self.request("tools/list") or {}).get("tools", [])

    def call_tool(self, name: str, arguments: Optional[dict] = None) -> dict:
        return self.request("tools/call", {"name": name, "arguments": arguments or {}}) or {}

    def list_resources(self) -> List[dict]:
        return (self.request("resources/list") or {}).get("resources", [])

    def read_resource(self, uri: str) -> dict:
        return self.request("resources/read", {"uri": uri}) or {}

    def list_prompts(self) -> List[dict]:
        return (self.request("prompts/list") or {}).get("prompts", [])

    def get_prompt(self, name: str, arguments: Optional[dict] = None) -> dict:
        return self.request("prompts/get", {"name": name, "arguments": arguments or {}}) or {}

    def close(self) -> None:
        if self._closed:
            return
        self._closed = True
        if self.proc is not None:
            if self.proc.poll() is None:
                try:
                    self.proc.stdin.close()
                    self.proc.wait(timeout=5)
                except Exception:
                    self.proc.kill()
            return
        try:
            if self.transport == "http" and self.session_id:
                self._http.delete(self.url, headers={**self.headers, "Mcp-Session-Id": self.session_id},
                                  timeout=self.timeout_s)
            if self.transport == "sse":
                # wake the reader thread (blocked in a read) by shutting the socket down; closing the
                # response while it reads would block
                import socket
                conn = getattr(self._sse.raw, "connection", None) or getattr(self._sse.raw, "_connection", None)
                sock = getattr(conn, "sock", None)
                if sock is not None:
                    sock.shutdown(socket.SHUT_RDWR)
        except Exception:
            pass


def tool_text(result: dict) -> str:
    """The text blocks of a ``tools/call`` result, joined."""
    return "\n".join(b.get("text", "") for b in result.get("content", []) if b.get("type") == "text")


class MCPRegistry:
    """Named MCP server connections; tool names are exposed as ``<server>__<tool>``."""

    SEP = "__"

    def __init__(self):
        self.clients: Dict[str, MCPClient] = {}

    def connect(self, name: str, command: Optional[List[str]] = None, timeout_s: float = 30.0,
                url: Optional[str] = None, transport: str = "stdio", headers: Optional[dict] = None) -> dict:
        if self.SEP in name or not name:
            raise ValueError(f"server name must be non-empty and must not contain {self.SEP!r}")
        self.disconnect(name)
        c = MCPClient(command, timeout_s, url=url, transport=transport if url else "stdio", headers=headers)
        try:
            info = c.initialize()
        except Exception:
            c.close()
            raise
        self.clients[name] = c
        return info

    def disconnect(self, name: str) -> bool:
        c = self.clients.pop(name, None)
        if c is not None:
            c.close()
        return c is not None

    def openai_tools(self) -> List[dict]:
        out = []
        for sname, c in self.clients.items():
            for t in c.list_tools():
                out.append({"type": "function", "function": {
                    "name": f"{sname}{self.SEP}{t['name']}", "description": t.get("description", ""),
                    "parameters": t.get("inputSchema") or {"type": "object", "properties": {}}}})
        return out

    def call(self, qualified: str, arguments: Optional[dict] = None) -> dict:
        sname, _, tname = qualified.partition(self.SEP)
        c = self.clients.get(sname)
        if c is None or not tname:
            raise KeyError(f"unknown MCP tool {qualified!r}")
        return c.call_tool(tname, arguments)

    def close(self) -> None:
        for n in list(self.clients):
            self.disconnect(n)
