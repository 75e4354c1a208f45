"""Model Context Protocol client (stdio transport) and registry of connected MCP servers.

Reference behaviour: plugins/gollek-plugin-mcp/…/mcp/dto/MCPConnection.java:82-170 (``initialize``
with the client's protocol version and capabilities, then ``notifications/initialized``,
``tools/list``), MCPToolExecutor / MCPResourceProvider / MCPPromptProvider (``tools/call``,
``resources/list`` + ``resources/read``, ``prompts/list`` + ``prompts/get``) and StdioTransport
(the server runs as a child process; JSON-RPC 2.0 messages, one per line, on its stdin / stdout).
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


class MCPClient:
    def __init__(self, command: List[str], timeout_s: float = 30.0, env: Optional[dict] = None):
        self.timeout_s = timeout_s
        self.proc = subprocess.Popen(command, stdin=subprocess.PIPE, stdout=subprocess.PIPE,
                                     stderr=subprocess.DEVNULL, text=True, bufsize=1, env=env)
        self._q: "queue.Queue[dict]" = queue.Queue()
        self._next_id = 1
        self._lock = threading.Lock()
        self.server_info: dict = {}
        self.protocol_version: Optional[str] = None
        threading.Thread(target=self._reader, daemon=True).start()

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

    def _send(self, msg: dict) -> None:
        if self.proc.poll() is not None:
            raise MCPError("MCP server exited")
        self.proc.stdin.write(json.dumps(msg) + "\n")
        self.proc.stdin.flush()

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
        if self.proc.poll() is None:
            try:
                self.proc.stdin.close()
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()


def tool_text(result: dict) -> str:
    """The text blocks of a ``tools/call`` result, joined."""
    return "\n".join(b.get("text", "") for b in result.get("content", []) if b.get("type") == "text")


class MCPRegistry:
    """Named MCP server connections; tool names are exposed as ``<server>__<tool>``."""

    SEP = "__"

    def __init__(self):
        self.clients: Dict[str, MCPClient] = {}

    def connect(self, name: str, command: List[str], timeout_s: float = 30.0) -> dict:
        if self.SEP in name or not name:
            raise ValueError(f"server name must be non-empty and must not contain {self.SEP!r}")
        self.disconnect(name)
        c = MCPClient(command, timeout_s)
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
