"""A minimal MCP server over stdio for the client tests: tools ``add`` and ``echo``, one resource and
one prompt. One JSON-RPC message per line."""
import json
import sys

TOOLS = [{"name": "add", "description": "add two integers",
          "inputSchema": {"type": "object", "properties": {"a": {"type": "integer"}, "b": {"type": "integer"}},
                          "required": ["a", "b"]}},
         {"name": "echo", "description": "echo text", "inputSchema": {"type": "object",
                                                                       "properties": {"text": {"type": "string"}}}}]


def handle(req):
    """The JSON-RPC reply to one request (None for a notification)."""
    m, mid, p = req.get("method"), req.get("id"), req.get("params") or {}
    if mid is None:
        return None

    def ok(result):
        return {"jsonrpc": "2.0", "id": mid, "result": result}

    def err(code, message):
        return {"jsonrpc": "2.0", "id": mid, "error": {"code": code, "message": message}}

    if m == "initialize":
        return ok({"protocolVersion": p.get("protocolVersion"), "capabilities": {"tools": {}},
                   "serverInfo": {"name": "fake", "version": "1"}})
    if m == "tools/list":
        return ok({"tools": TOOLS})
    if m == "tools/call":
        a = p.get("arguments", {})
        if p.get("name") == "add":
            return ok({"content": [{"type": "text", "text": str(int(a["a"]) + int(a["b"]))}], "isError": False})
        if p.get("name") == "echo":
            return ok({"content": [{"type": "text", "text": a.get("text", "")}]})
        return err(-32602, "unknown tool")
    if m == "resources/list":
        return ok({"resources": [{"uri": "mem://readme", "name": "readme"}]})
    if m == "resources/read":
        return ok({"contents": [{"uri": p["uri"], "text": "hello from the resource"}]})
    if m == "prompts/list":
        return ok({"prompts": [{"name": "greet", "arguments": [{"name": "who"}]}]})
    if m == "prompts/get":
        who = p.get("arguments", {}).get("who", "you")
        return ok({"messages": [{"role": "user", "content": {"type": "text", "text": f"Say hi to {who}"}}]})
    return err(-32601, "method not found")


if __name__ == "__main__":
    for line in sys.stdin:
        req = json.loads(line)
        rep = handle(req)
        if rep is None:
            continue  # notification
        sys.stdout.write(json.dumps({"jsonrpc": "2.0", "method": "notifications/message",
                                     "params": {"level": "info"}}) + "\n")
        sys.stdout.write(json.dumps(rep) + "\n")
        sys.stdout.flush()
