"""Model Context Protocol adapter: the gym operations as MCP tools over stdio (JSON-RPC 2.0).

    python -m nexttransformer_b200.gym mcp --credential credential.json

``tools/list`` is generated from the operation table, so every HTTP operation is a tool with the
same input schema; ``tools/call`` forwards to the HTTP API and returns the JSON result as text
content (``isError`` set on a gym error).  One JSON-RPC message per line.
"""
import json
import sys

from nexttransformer_b200.gym.contract import OPERATIONS, SCHEMA_VERSION, GymError

PROTOCOL = "2024-11-05"


def handle(message, call):
    """The JSON-RPC response to ``message`` (None for a notification); ``call(op, params)`` runs a tool."""
    mid, method, params = message.get("id"), message.get("method"), message.get("params") or {}
    if mid is None:
        return None
    if method == "initialize":
        result = dict(protocolVersion=PROTOCOL, capabilities={"tools": {}},
                      serverInfo=dict(name="nexttransformer_b200-gym", version=SCHEMA_VERSION))
    elif method == "ping":
        result = {}
    elif method == "tools/list":
        result = dict(tools=[dict(name=n, description=op["description"], inputSchema=op["inputSchema"])
                             for n, op in OPERATIONS.items()])
    elif method == "tools/call":
        name, args = params.get("name"), params.get("arguments") or {}
        try:
            out = call(name, args)
            result = dict(content=[dict(type="text", text=json.dumps(out))], isError=False)
        except GymError as e:
            result = dict(content=[dict(type="text", text=json.dumps(dict(code=e.code, message=e.message)))],
                          isError=True)
    else:
        return dict(jsonrpc="2.0", id=mid, error=dict(code=-32601, message=f"unknown method {method}"))
    return dict(jsonrpc="2.0", id=mid, result=result)


def serve(call, stdin=sys.stdin, stdout=sys.stdout):
    for line in stdin:
        line = line.strip()
        if not line:
            continue
        try:
            message = json.loads(line)
        except json.JSONDecodeError:
            reply = dict(jsonrpc="2.0", id=None, error=dict(code=-32700, message="parse error"))
        else:
            reply = handle(message, call)
        if reply is not None:
            stdout.write(json.dumps(reply) + "\n")
            stdout.flush()
