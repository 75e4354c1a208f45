"""A minimal MCP server over stdio for the client tests: tools ``add`` and ``echo``, one resource and
one prompt. One JSON-RPC message per line."""
import json
import sys

TOOLS = [{"name": "add", "description": "add two integers",
          "inputSchema": {"type": "object", "properties": {"a": {"type": "integer"}, "b": {"type": "integer"}},
                          "required": ["a", "b"]}},
         {"name": "echo", "description": "echo text", "inputSchema": {"type": "object",
                                                                       "properties": {"text": {"type": "string"}}}}]


def reply(mid, result=None, error=None):
    msg = {"jsonrpc": "2.0", "id": mid}
    msg.update({"error": error} if error else {"result": result})
    sys.stdout.write(json.dumps(msg) + "\n")
    sys.stdout.flush()


for line in sys.stdin:
    req = json.loads(line)
    m, mid, p = req.get("method"), req.get("id"), req.get("params") or {}
    if mid is None:
        continue  # notification
    sys.stdout.write(json.dumps({"jsonrpc": "2.0", "method": "notifications/message", "params": {"level": "info"}}) + "\n")
    if m == "initialize":
        reply(mid, {"protocolVersion": p.get("protocolVersion"), "capabilities": {"tools": {}},
                    "serverInfo": {"name": "fake", "version": "1"}})
    elif m == "tools/list":
        reply(mid, {"tools": TOOLS})
    elif m == "tools/call":
        a = p.get("arguments", {})
        if p.get("name") == "add":
            reply(mid, {"content": [{"type": "text", "text": str(int(a["a"]) + int(a["b"]))}], "isError": False})
        elif p.get("name") == "echo":
            reply(mid, {"content": [{"type": "text", "text": a.get("text", "")}]})
        else:
            reply(mid, error={"code": -32602, "message": "unknown tool"})
    elif m == "resources/list":
        reply(mid, {"resources": [{"uri": "mem://readme", "name": "readme"}]})
    elif m == "resources/read":
        reply(mid, {"contents": [{"uri": p["uri"], "text": "hello from the resource"}]})
    elif m == "prompts/list":
        reply(mid, {"prompts": [{"name": "greet", "arguments": [{"name": "who"}]}]})
    elif m == "prompts/get":
        who = p.get("arguments", {}).get("who", "you")
        reply(mid, {"messages": [{"role": "user", "content": {"type": "text", "text": f"Say hi to {who}"}}]})
    else:
        reply(mid, error={"code": -32601, "message": "method not found"})
