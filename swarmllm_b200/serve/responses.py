"""OpenAI Responses API on the local engine.

  POST   /v1/responses                  create (stream / background / store)
  GET    /v1/responses/{id}             the stored object; ?stream=true replays a
                                        background run's events (after
                                        ?starting_after=N) and follows it live
  DELETE /v1/responses/{id}
  POST   /v1/responses/{id}/cancel      cancel a background run in flight
  GET    /v1/responses/{id}/input_items paginated (limit, order, after)

A request is translated into a chat conversation: `instructions` become the
system message, `previous_response_id` prepends the stored conversation of
that response (its input and output; its instructions are not carried over),
and input items map to messages (message, function_call,
function_call_output).  Function tools go through the same tool prompt and
parser as chat completions and come back as `function_call` output items.
Generation produces the typed event sequence (response.created ...
response.output_text.delta ... response.completed); a non-streaming request
consumes the same sequence and returns the final object.

`store` (default true) persists the response, its input items and its
conversation in SQLite (a file given at start-up, else in memory).
`background=true` runs the generation as a task: without `stream` the reply
is 202 with a Location header; with `stream` the events also go to a replay
buffer that GET ?stream=true serves from any sequence number.

Reference behaviour: src/api/openai/responses/ (mod.rs create/cancel/delete/
input_items, store.rs, background.rs replay buffer, stream.rs event order,
translate.rs item <-> chat mapping).
"""
from __future__ import annotations

import asyncio
import base64
import json
import sqlite3
import threading
import time
import uuid

from fastapi import Request  # module level: route annotations resolve from globals

MAX_INPUT_ITEMS = 1024
MAX_INSTRUCTIONS_BYTES = 2 << 20
MAX_PREV_ID_LEN = 64


def _hex(n=24) -> str:
    return uuid.uuid4().hex[:n]


class ResponseStore:
    """Responses with their input items and conversation, in SQLite."""

    def __init__(self, path: str | None = None):
        self.db = sqlite3.connect(path or ":memory:", check_same_thread=False)
        self.lock = threading.Lock()
        with self.lock:
            self.db.execute("CREATE TABLE IF NOT EXISTS responses (id TEXT PRIMARY KEY, created REAL, "
                            "obj TEXT, items TEXT, convo TEXT)")
            self.db.commit()

    def put(self, obj: dict, items: list, convo: list):
        with self.lock:
            self.db.execute("INSERT OR REPLACE INTO responses VALUES (?, ?, ?, ?, ?)",
                            (obj["id"], time.time(), json.dumps(obj), json.dumps(items), json.dumps(convo)))
            self.db.commit()

    def get(self, rid: str):
        with self.lock:
            row = self.db.execute("SELECT obj, items, convo FROM responses WHERE id = ?", (rid,)).fetchone()
        return None if row is None else tuple(json.loads(x) for x in row)

    def delete(self, rid: str) -> bool:
        with self.lock:
            n = self.db.execute("DELETE FROM responses WHERE id = ?", (rid,)).rowcount
            self.db.commit()
        return n > 0

    def prune(self, older_than_s: float | None = None, keep: int | None = None) -> tuple[int, int]:
        """Delete stored responses older than `older_than_s` seconds and/or all
        but the newest `keep`; returns (removed, left)."""
        with self.lock:
            n = 0
            if older_than_s is not None:
                n += self.db.execute("DELETE FROM responses WHERE created < ?",
                                     (time.time() - older_than_s,)).rowcount
            if keep is not None:
                n += self.db.execute(
                    "DELETE FROM responses WHERE id NOT IN "
                    "(SELECT id FROM responses ORDER BY created DESC LIMIT ?)", (max(0, keep),)).rowcount
            self.db.commit()
            left = self.db.execute("SELECT COUNT(*) FROM responses").fetchone()[0]
        return n, left


class _Run:
    """A background run: its task, its event log and waiters."""

    def __init__(self, obj: dict):
        self.obj = obj
        self.events: list[dict] = []
        self.done = False
        self.task: asyncio.Task | None = None
        self.changed = asyncio.Event()

    def add(self, ev: dict):
        self.events.append(ev)
        self.changed.set()

    async def follow(self, after: int):
        """Events with sequence_number > after, then live ones until the end."""
        i = 0
        while True:
            while i < len(self.events):
                ev = self.events[i]
                i += 1
                if ev["sequence_number"] > after:
                    yield ev
            if self.done:
                return
            self.changed.clear()
            if i < len(self.events):
                continue
            await self.changed.wait()


def _item_text(content) -> str:
    if isinstance(content, str):
        return content
    out = []
    for p in content or []:
        if not isinstance(p, dict):
            continue
        t = p.get("type")
        if t in ("input_text", "output_text", "text"):
            out.append(p.get("text", ""))
        elif t == "input_file":
            data = p.get("file_data", "")
            if "," in data and data.startswith("data:"):
                data = data.split(",", 1)[1]
            try:
                out.append(base64.b64decode(data).decode("utf-8"))
            except (ValueError, UnicodeDecodeError):
                raise ValueError("input_file must be UTF-8 text (base64 file_data)")
        elif t == "input_image":
            raise ValueError("this model takes no image input")
    return "".join(out)


def items_of(inp) -> list[dict]:
    """The request's input as a list of items, each with an id."""
    if isinstance(inp, str):
        inp = [{"type": "message", "role": "user", "content": [{"type": "input_text", "text": inp}]}]
    if not isinstance(inp, list):
        raise ValueError("input must be a string or a list of items")
    if len(inp) > MAX_INPUT_ITEMS:
        raise ValueError(f"at most {MAX_INPUT_ITEMS} input items")
    items = []
    for it in inp:
        if not isinstance(it, dict):
            raise ValueError("input items must be objects")
        it = dict(it)
        it.setdefault("type", "message")
        if it["type"] == "message":
            c = it.get("content", "")
            if isinstance(c, str):
                it["content"] = [{"type": "input_text", "text": c}]
        it.setdefault("id", {"message": "msg_", "function_call": "fc_"}.get(it["type"], "item_") + _hex())
        items.append(it)
    return items


def messages_of(items: list[dict]) -> list[dict]:
    msgs = []
    for it in items:
        t = it["type"]
        if t == "message":
            role = it.get("role", "user")
            c = it.get("content")
            has_image = isinstance(c, list) and any(isinstance(p, dict) and p.get("type") == "input_image"
                                                    for p in c)
            msgs.append({"role": "system" if role == "developer" else role,
                         "content": c if has_image else _item_text(c)})
        elif t == "function_call":
            msgs.append({"role": "assistant", "content": "", "tool_calls": [
                {"id": it.get("call_id"), "function": {"name": it.get("name"),
                                                       "arguments": it.get("arguments", "{}")}}]})
        elif t == "function_call_output":
            out = it.get("output", "")
            msgs.append({"role": "tool", "tool_call_id": it.get("call_id", ""),
                         "content": out if isinstance(out, str) else json.dumps(out)})
        else:
            raise ValueError(f"unsupported input item type {t!r}")
    return msgs


def register(app, S, store_path: str | None = None):
    from fastapi.responses import JSONResponse, StreamingResponse

    from .api import ApiError
    from .tools import tools_from_openai

    store = ResponseStore(store_path)
    runs: dict[str, _Run] = {}
    app.state.response_store = store

    def sse(ev: dict) -> str:
        return f"event: {ev['type']}\ndata: {json.dumps(ev)}\n\n"

    async def produce(obj: dict, ids, sp, stops, tools, lora, items, convo, persist: bool,
                      images=None):
        """The typed event sequence of one generation; stores the result."""
        seq = [0]

        def ev(kind, **kw):
            seq[0] += 1
            return dict(type=kind, sequence_number=seq[0], **kw)

        yield ev("response.created", response=dict(obj))
        yield ev("response.in_progress", response=dict(obj))
        msg_id = "msg_" + _hex()
        opened = False
        text = ""
        try:
            async for e in S.stream(ids, sp, stops, tools, lora, images):
                delta = e[1] if e[0] == "text" else e[1].rest
                if delta or (e[0] == "done" and not opened and not e[1].calls):
                    if not opened:
                        opened = True
                        yield ev("response.output_item.added", output_index=0, item={
                            "type": "message", "id": msg_id, "status": "in_progress",
                            "role": "assistant", "content": []})
                        yield ev("response.content_part.added", item_id=msg_id, output_index=0,
                                 content_index=0, part={"type": "output_text", "text": "", "annotations": []})
                    if delta:
                        text += delta
                        yield ev("response.output_text.delta", item_id=msg_id, output_index=0,
                                 content_index=0, delta=delta)
                if e[0] != "done":
                    continue
                r = e[1]
                output = []
                if opened:
                    part = {"type": "output_text", "text": r.text, "annotations": []}
                    item = {"type": "message", "id": msg_id, "status": "completed",
                            "role": "assistant", "content": [part]}
                    yield ev("response.output_text.done", item_id=msg_id, output_index=0,
                             content_index=0, text=r.text)
                    yield ev("response.content_part.done", item_id=msg_id, output_index=0,
                             content_index=0, part=part)
                    yield ev("response.output_item.done", output_index=0, item=item)
                    output.append(item)
                for c in r.calls:
                    k = len(output)
                    item = {"type": "function_call", "id": "fc_" + _hex(), "call_id": c.id,
                            "name": c.name, "arguments": c.arguments, "status": "completed"}
                    yield ev("response.output_item.added", output_index=k,
                             item=dict(item, arguments="", status="in_progress"))
                    yield ev("response.function_call_arguments.delta", item_id=item["id"],
                             output_index=k, delta=c.arguments)
                    yield ev("response.function_call_arguments.done", item_id=item["id"],
                             output_index=k, arguments=c.arguments)
                    yield ev("response.output_item.done", output_index=k, item=item)
                    output.append(item)
                obj.update(output=output, output_text=r.text,
                           usage={"input_tokens": r.n_prompt, "output_tokens": r.n_out,
                                  "total_tokens": r.n_prompt + r.n_out})
                if r.finish == "length":
                    obj.update(status="incomplete", incomplete_details={"reason": "max_output_tokens"})
                else:
                    obj.update(status="completed")
                asst = {"role": "assistant", "content": r.text}
                if r.calls:
                    asst["tool_calls"] = [c.openai() for c in r.calls]
                if persist:
                    store.put(obj, items, convo + [asst])
                yield ev("response.completed" if obj["status"] == "completed" else "response.incomplete",
                         response=dict(obj))
                return
        except asyncio.CancelledError:
            obj.update(status="cancelled")
            if persist:
                store.put(obj, items, convo)
            raise
        except ApiError as e:
            obj.update(status="failed", error={"code": "server_error", "message": e.message})
            if persist:
                store.put(obj, items, convo)
            yield ev("response.failed", response=dict(obj))

    @app.post("/v1/responses")
    async def create_response(request: Request):
        try:
            body = await request.json()
        except ValueError:
            raise ApiError(400, "request body is not valid JSON")
        if not isinstance(body, dict) or "input" not in body:
            raise ApiError(400, "input is required")
        instr = body.get("instructions")
        prev = body.get("previous_response_id")
        if instr is not None and (not isinstance(instr, str) or len(instr.encode()) > MAX_INSTRUCTIONS_BYTES):
            raise ApiError(400, "instructions must be a string of at most 2 MiB")
        if prev is not None and (not isinstance(prev, str) or len(prev) > MAX_PREV_ID_LEN):
            raise ApiError(400, "previous_response_id is not a response id")
        try:
            items = items_of(body["input"])
            tools = tools_from_openai(body.get("tools"))
            convo = []
            if prev:
                got = store.get(prev)
                if got is None:
                    raise ApiError(404, f"previous response {prev} not found")
                convo = got[2]
            convo = convo + messages_of(items)
        except ValueError as e:
            raise ApiError(400, str(e))
        msgs = ([{"role": "system", "content": instr}] if instr else []) + convo
        fmt = (body.get("text") or {}).get("format")
        if fmt and fmt.get("type") == "json_schema":
            fmt = {"type": "json_schema", "json_schema": {"schema": fmt.get("schema")}}
        ids, tools, images = S.prepare(msgs, tools, body.get("tool_choice"), fmt)
        sp = S.params(body, S.prompt_len(ids, images), fmt)
        lora = S.lora_of(body)
        persist = body.get("store", True) is not False
        background, stream = bool(body.get("background")), bool(body.get("stream"))
        rid = "resp_" + _hex(32)
        obj = {"id": rid, "object": "response", "created_at": int(time.time()),
               "status": "queued" if background else "in_progress",
               "model": body.get("model") or S.model_name, "output": [], "output_text": "",
               "instructions": instr, "previous_response_id": prev, "store": persist,
               "background": background, "error": None, "incomplete_details": None,
               "max_output_tokens": sp.max_tokens, "temperature": sp.temperature, "top_p": sp.top_p,
               "tools": body.get("tools") or [], "tool_choice": body.get("tool_choice", "auto"),
               "metadata": body.get("metadata") or {}, "usage": None}
        gen = produce(obj, ids, sp, S.stops(body), tools, lora, items, convo, persist, images)

        if background:
            run = runs[rid] = _Run(obj)
            if persist:
                store.put(obj, items, convo)

            async def drive():
                try:
                    async for e in gen:
                        run.add(e)
                except asyncio.CancelledError:
                    run.add({"type": "response.cancelled", "sequence_number":
                             (run.events[-1]["sequence_number"] + 1) if run.events else 1,
                             "response": dict(obj)})
                finally:
                    run.done = True
                    run.changed.set()
            run.task = asyncio.get_running_loop().create_task(drive())
            if stream:
                async def tail():
                    async for e in run.follow(0):
                        yield sse(e)
                return StreamingResponse(tail(), media_type="text/event-stream")
            return JSONResponse(dict(obj), status_code=202, headers={"location": f"/v1/responses/{rid}"})
        if stream:
            async def live():
                async for e in gen:
                    yield sse(e)
            return StreamingResponse(live(), media_type="text/event-stream")
        async for _ in gen:
            pass
        if obj["status"] == "failed":
            raise ApiError(500, obj["error"]["message"], "server_error")
        return JSONResponse(obj)

    def current(rid: str):
        run = runs.get(rid)
        if run is not None:
            return run.obj
        got = store.get(rid)
        return None if got is None else got[0]

    @app.get("/v1/responses/{rid}")
    async def get_response(rid: str, request: Request):
        qp = request.query_params
        if qp.get("stream") in ("true", "1"):
            run = runs.get(rid)
            if run is None:
                raise ApiError(400 if current(rid) else 404,
                               "only background responses can be streamed again")
            after = int(qp.get("starting_after", "0") or 0)

            async def tail():
                async for e in run.follow(after):
                    yield sse(e)
            return StreamingResponse(tail(), media_type="text/event-stream")
        obj = current(rid)
        if obj is None:
            raise ApiError(404, f"response {rid} not found")
        return JSONResponse(obj)

    @app.delete("/v1/responses/{rid}")
    async def delete_response(rid: str):
        run = runs.pop(rid, None)
        if run is not None and run.task is not None and not run.done:
            run.task.cancel()
        ok = store.delete(rid)
        if not ok and run is None:
            raise ApiError(404, f"response {rid} not found")
        return {"id": rid, "object": "response.deleted", "deleted": True}

    @app.post("/v1/responses/{rid}/cancel")
    async def cancel_response(rid: str):
        run = runs.get(rid)
        if run is None:
            if current(rid) is None:
                raise ApiError(404, f"response {rid} not found")
            raise ApiError(400, "only background responses can be cancelled")
        if not run.done and run.task is not None:
            run.task.cancel()
            try:
                await run.task
            except asyncio.CancelledError:
                pass
        return JSONResponse(run.obj)

    @app.get("/v1/responses/{rid}/input_items")
    async def list_input_items(rid: str, request: Request):
        got = store.get(rid)
        if got is None:
            raise ApiError(404, f"response {rid} not found")
        qp = request.query_params
        try:
            limit = max(1, min(100, int(qp.get("limit", "20"))))
        except ValueError:
            raise ApiError(400, "limit must be an integer")
        order = qp.get("order", "desc")
        if order not in ("asc", "desc"):
            raise ApiError(400, "order must be asc or desc")
        items = list(got[1])
        if order == "desc":
            items.reverse()
        after = qp.get("after")
        if after:
            k = next((i for i, it in enumerate(items) if it.get("id") == after), None)
            if k is None:
                raise ApiError(400, f"unknown cursor {after}")
            items = items[k + 1:]
        page = items[:limit]
        return {"object": "list", "data": page, "first_id": page[0]["id"] if page else None,
                "last_id": page[-1]["id"] if page else None, "has_more": len(items) > limit}
