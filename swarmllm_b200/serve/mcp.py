"""Model Context Protocol server (Streamable HTTP transport) at /mcp.

POST carries one JSON-RPC 2.0 message.  Requests get a JSON-RPC reply;
notifications (no id) get 202 with an empty body.  GET (a server-to-client
stream) is 405, since this server never initiates messages; DELETE (end of
session) is 200.  Bodies that are not JSON get -32700 with a null id; JSON
that is not a request object gets -32600; unknown methods -32601.

Methods: initialize (protocol-version negotiation), ping, tools/list,
tools/call, resources/list, resources/read.  Tools run on this node's
engine, so a batch of prompts is served by continuous batching:

  chat           one prompt (or messages) -> text
  models         the base model and its LoRA adapters
  compare        one prompt on several of those models, side by side
  batch_prompts  many independent prompts at once (optionally one model each)
  node_info      engine and device status

Resources: swarmllm://status, swarmllm://models, swarmllm://peers.

Reference behaviour: src/api/mcp/mod.rs (handle_mcp, versions, notification
202, error codes), tools_list.rs, tools.rs, resources.rs.
"""
from __future__ import annotations

import asyncio
import json

from fastapi import Request  # module level: route annotations resolve from globals

PROTOCOL_VERSIONS = ("2025-11-25", "2025-06-18", "2025-03-26", "2024-11-05")
PARSE_ERROR, INVALID_REQUEST, METHOD_NOT_FOUND, INVALID_PARAMS, INTERNAL = (
    -32700, -32600, -32601, -32602, -32603)
RESOURCE_NOT_FOUND = -32002
MAX_PROMPT_BYTES = 4 << 20
MAX_BATCH = 64

INSTRUCTIONS = ("Local LLM inference on this node's GPUs. Use these tools to run a prompt on the "
                "served model (or one of its LoRA adapters), compare adapters side by side, or run "
                "many independent prompts at once in one batch.")


def _schema(props: dict, required=()) -> dict:
    return {"type": "object", "properties": props, "required": list(required)}


_GEN = {"max_tokens": {"type": "integer", "description": "maximum tokens to generate"},
        "temperature": {"type": "number"}, "system": {"type": "string"}}

TOOLS = [
    {"name": "chat", "description": "Run one prompt on the served model (or a LoRA adapter).",
     "inputSchema": _schema({"prompt": {"type": "string"}, "model": {"type": "string"},
                             "messages": {"type": "array"}, **_GEN})},
    {"name": "models", "description": "List the models this node serves (base and LoRA adapters).",
     "inputSchema": _schema({})},
    {"name": "compare", "description": "Run one prompt on several models and return each answer.",
     "inputSchema": _schema({"prompt": {"type": "string"},
                             "models": {"type": "array", "items": {"type": "string"}}, **_GEN},
                            ["prompt"])},
    {"name": "batch_prompts", "description": "Run many independent prompts concurrently.",
     "inputSchema": _schema({"tasks": {"type": "array", "items": _schema(
         {"id": {"type": "string"}, "prompt": {"type": "string"}, "model": {"type": "string"},
          "max_tokens": {"type": "integer"}}, ["prompt"])}, **_GEN}, ["tasks"])},
    {"name": "node_info", "description": "Engine, cache and device status of this node.",
     "inputSchema": _schema({})},
]

RESOURCES = [
    {"uri": "swarmllm://status", "name": "Node Status", "mimeType": "application/json",
     "description": "Engine status: running and waiting requests, KV pages, uptime"},
    {"uri": "swarmllm://models", "name": "Available Models", "mimeType": "application/json",
     "description": "The served model and its LoRA adapters"},
    {"uri": "swarmllm://peers", "name": "Connected Peers", "mimeType": "application/json",
     "description": "Pipeline peers of this node (none when serving on one node)"},
]


def _ok(rid, result) -> dict:
    return {"jsonrpc": "2.0", "id": rid, "result": result}


def _err(rid, code: int, message: str) -> dict:
    return {"jsonrpc": "2.0", "id": rid, "error": {"code": code, "message": message}}


class ToolError(Exception):
    pass


def register(app, S):
    from fastapi.responses import JSONResponse, Response

    async def gen(prompt: str | None, args: dict, model: str | None = None, messages=None) -> dict:
        if prompt is not None and len(prompt.encode()) > MAX_PROMPT_BYTES:
            raise ToolError("prompt over 4 MiB")
        msgs = list(messages or [])
        if prompt is not None:
            msgs.append({"role": "user", "content": prompt})
        if not msgs:
            raise ToolError("prompt or messages is required")
        if args.get("system"):
            msgs.insert(0, {"role": "system", "content": str(args["system"])})
        body = {"max_tokens": args.get("max_tokens", 256), "temperature": args.get("temperature", 0.0),
                "model": model}
        ids, _, _ = S.prepare(msgs)
        sp = S.params(body, len(ids))
        r = await S.run(ids, sp, [], None, S.lora_of(body))
        return {"model": model or S.model_name, "text": r.text, "finish_reason": r.finish,
                "usage": {"prompt_tokens": r.n_prompt, "completion_tokens": r.n_out}}

    def check_model(m):
        if m and m not in S.models() and S.lora_of({"model": m}) is None:
            raise ToolError(f"unknown model {m!r}; see the models tool")

    async def call_tool(name: str, args: dict) -> dict:
        if name == "chat":
            check_model(args.get("model"))
            out = await gen(args.get("prompt"), args, args.get("model"), args.get("messages"))
            return {"content": [{"type": "text", "text": out["text"]}], "structuredContent": out,
                    "isError": False}
        if name == "models":
            data = {"models": S.models()}
            return {"content": [{"type": "text", "text": json.dumps(data)}], "structuredContent": data,
                    "isError": False}
        if name == "compare":
            models = args.get("models") or S.models()
            if not isinstance(models, list) or len(models) > MAX_BATCH:
                raise ToolError(f"models must be a list of at most {MAX_BATCH}")
            for m in models:
                check_model(m)
            outs = await asyncio.gather(*[gen(args.get("prompt"), args, m) for m in models])
            text = "\n\n".join(f"## {o['model']}\n{o['text']}" for o in outs)
            return {"content": [{"type": "text", "text": text}], "structuredContent": {"results": outs},
                    "isError": False}
        if name == "batch_prompts":
            tasks = args.get("tasks")
            if not isinstance(tasks, list) or not tasks or len(tasks) > MAX_BATCH:
                raise ToolError(f"tasks must be a list of 1 to {MAX_BATCH} entries")
            for t in tasks:
                if not isinstance(t, dict) or not isinstance(t.get("prompt"), str):
                    raise ToolError("every task needs a prompt string")
                if len(str(t.get("id", ""))) > 256:
                    raise ToolError("task id over 256 characters")
                check_model(t.get("model"))
            outs = await asyncio.gather(*[
                gen(t["prompt"], dict(args, **({"max_tokens": t["max_tokens"]} if "max_tokens" in t else {})),
                    t.get("model")) for t in tasks])
            res = [dict(o, id=str(t.get("id", i))) for i, (t, o) in enumerate(zip(tasks, outs))]
            return {"content": [{"type": "text", "text": json.dumps(res)}],
                    "structuredContent": {"results": res}, "isError": False}
        if name == "node_info":
            info = node_info()
            return {"content": [{"type": "text", "text": json.dumps(info)}], "structuredContent": info,
                    "isError": False}
        raise KeyError(name)

    def node_info() -> dict:
        info = dict(S.status()) if hasattr(S, "status") else {}
        try:
            import torch
            if torch.cuda.is_available():
                info["devices"] = [{"index": i, "name": torch.cuda.get_device_name(i),
                                    "memory_gb": round(torch.cuda.get_device_properties(i).total_memory / 2**30, 1)}
                                   for i in range(torch.cuda.device_count())]
        except Exception:
            pass
        return info

    def read_resource(uri: str):
        if uri == "swarmllm://status":
            return node_info()
        if uri == "swarmllm://models":
            return {"models": S.models()}
        if uri == "swarmllm://peers":
            return {"peers": []}
        return None

    async def handle(msg: dict):
        rid = msg.get("id")
        method = msg.get("method")
        params = msg.get("params") or {}
        if method == "initialize":
            want = params.get("protocolVersion")
            ver = want if want in PROTOCOL_VERSIONS else PROTOCOL_VERSIONS[0]
            return _ok(rid, {"protocolVersion": ver,
                             "capabilities": {"tools": {"listChanged": False},
                                              "resources": {"listChanged": False, "subscribe": False}},
                             "serverInfo": {"name": "swarmllm_b200", "version": "0.1.0"},
                             "instructions": INSTRUCTIONS})
        if method == "ping":
            return _ok(rid, {})
        if method == "tools/list":
            return _ok(rid, {"tools": TOOLS})
        if method == "tools/call":
            name = params.get("name")
            args = params.get("arguments") or {}
            if not isinstance(args, dict):
                return _err(rid, INVALID_PARAMS, "arguments must be an object")
            try:
                return _ok(rid, await call_tool(name, args))
            except KeyError:
                return _err(rid, INVALID_PARAMS, f"unknown tool {str(name)[:64]!r}")
            except Exception as e:   # tool failures are results, not protocol errors
                msg_ = getattr(e, "message", None) or str(e)
                return _ok(rid, {"content": [{"type": "text", "text": msg_}], "isError": True})
        if method == "resources/list":
            return _ok(rid, {"resources": RESOURCES})
        if method == "resources/read":
            uri = params.get("uri", "")
            data = read_resource(uri)
            if data is None:
                return _err(rid, RESOURCE_NOT_FOUND, f"unknown resource {str(uri)[:64]}")
            return _ok(rid, {"contents": [{"uri": uri, "mimeType": "application/json",
                                           "text": json.dumps(data)}]})
        if method == "sampling/createMessage":
            return _err(rid, METHOD_NOT_FOUND, "sampling/createMessage is not offered: this is a "
                                               "tools-only server; run inference with tools/call")
        shown = str(method)
        shown = shown if len(shown) <= 64 else shown[:64] + "..."
        return _err(rid, METHOD_NOT_FOUND, f"Method not found: {shown}")

    @app.post("/mcp")
    async def mcp_post(request: Request):
        raw = await request.body()
        try:
            msg = json.loads(raw)
        except ValueError as e:
            return JSONResponse(_err(None, PARSE_ERROR, f"Parse error: {e}"), status_code=400)
        if not isinstance(msg, dict) or msg.get("jsonrpc") != "2.0" or not isinstance(msg.get("method"), str):
            rid = msg.get("id") if isinstance(msg, dict) else None
            return JSONResponse(_err(rid, INVALID_REQUEST, "Invalid Request: expected one JSON-RPC 2.0 "
                                                          "request object"), status_code=400)
        if "id" not in msg or msg["id"] is None:     # a notification
            return Response(status_code=202)
        return JSONResponse(await handle(msg))

    @app.get("/mcp")
    async def mcp_get():
        return Response(status_code=405)

    @app.delete("/mcp")
    async def mcp_delete():
        return Response(status_code=200)
