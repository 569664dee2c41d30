"""OpenAI-, Anthropic- and MCP-compatible HTTP API on port 8800.

Routes (reference: src/api/server.rs:239-330, src/api/openai/mod.rs:319,
src/api/openai/streaming.rs:1431, src/api/anthropic/):
  POST /v1/chat/completions    (stream=true -> SSE chunks, data: [DONE]); tools,
                               tool_choice, response_format
  POST /v1/completions
  POST /v1/messages            (Anthropic Messages; tools -> tool_use blocks;
                               stream -> typed SSE events)
  POST /v1/responses, GET/DELETE /v1/responses/{id}, POST .../cancel,
  GET .../input_items          (OpenAI Responses API: serve/responses.py)
  POST/GET/DELETE /mcp         (Model Context Protocol server: serve/mcp.py)
  POST /v1/embeddings          (mean-pooled, L2-normalised input embeddings)
  GET  /v1/models              (the base model and every loaded LoRA adapter)
  GET  /v1/models/{id}, POST /v1/messages/count_tokens
  GET  /health, /health/ready, /metrics (Prometheus), /api/status, /v1/status
  POST /api/prefix/export, /api/prefix/import   (prefix-KV snapshots, engine/prefix_share.py)
  /api/admin/*                 (stats, performance, config, models, lora,
                               diagnostics, responses, storage: serve/admin.py)
  WS   /api/admin/ws           (status feed, one JSON message a second)

Auth, CORS, rate limits, security headers and the body-size cap are one ASGI
middleware (serve/middleware.py).  A request selects a LoRA adapter by naming
it as the model ("adapter" or "base:adapter").

The engine is single-threaded: ``AsyncEngine`` runs ``step()`` in a worker
thread, takes new requests from a queue between steps and hands each token
to the request's asyncio queue.  Continuous batching therefore happens
across HTTP requests automatically.
"""
from __future__ import annotations

import asyncio
import dataclasses
import itertools
import json
import os
import secrets
import queue
import threading
import time
import uuid
from dataclasses import dataclass, field

from fastapi import Request, WebSocket  # module level: route annotations resolve from globals

from ..engine.sampling import SamplingParams
from ..utils.logsetup import get_logger
from ..utils.metrics import Metrics
from .chat_template import render
from .tools import (ToolSpec, content_prefix_len, format_tool_prompt, parse_tool_calls,
                    tool_choice_forbids, tools_from_anthropic, tools_from_openai)


_log = get_logger("serve")


@dataclass
class _Sub:
    rid: int
    prompt: list
    params: SamplingParams
    q: asyncio.Queue
    loop: asyncio.AbstractEventLoop
    lora: str | None = None
    images: list | None = None


class AsyncEngine:
    """The engine on its own thread; HTTP handlers talk to it through queues.

    Readiness (`ready`) is withdrawn when a step raised, when the thread died,
    or while the loop is stalled: one step running, or submitted work left
    untouched, for more than `stall_s` seconds (default 300, env
    SWARMLLM_STALL_S).  A stall that ends gives readiness back.
    Reference behaviour: a dispatcher silent for 300 s withdraws the node's
    inference capability (docs/ARCHITECTURE.md:354-377)."""

    def __init__(self, engine, metrics: Metrics | None = None, stall_s: float | None = None):
        self.engine = engine
        self.metrics = metrics or Metrics()
        self.stall_s = float(os.environ.get("SWARMLLM_STALL_S", "300")) if stall_s is None else stall_s
        self._failed = False
        self._beat = time.monotonic()          # last pass of the loop
        self._step_since: float | None = None  # start of the step in progress
        self._stall_logged = False
        self._in: queue.Queue = queue.Queue()
        self._abort: queue.Queue = queue.Queue()
        self._calls: queue.Queue = queue.Queue()
        self._subs: dict[int, _Sub] = {}
        self._ids = itertools.count(1)
        self._wake = threading.Event()
        self._stop = False
        self._t = threading.Thread(target=self._run, daemon=True, name="engine")
        self._t.start()

    def submit(self, prompt_ids, params: SamplingParams, lora: str | None = None,
               images=None) -> tuple[int, asyncio.Queue]:
        rid = next(self._ids)
        q: asyncio.Queue = asyncio.Queue()
        self._in.put(_Sub(rid, list(prompt_ids), params, q, asyncio.get_running_loop(), lora,
                          images))
        self._wake.set()
        return rid, q

    def abort(self, rid: int):
        self._abort.put(rid)
        self._wake.set()

    async def call(self, fn):
        """Run fn(engine) on the engine thread between steps; returns its result."""
        loop = asyncio.get_running_loop()
        fut = loop.create_future()
        self._calls.put((fn, fut, loop))
        self._wake.set()
        return await fut

    def stalled(self) -> bool:
        now = time.monotonic()
        if self._step_since is not None and now - self._step_since > self.stall_s:
            return True
        return not self._in.empty() and now - self._beat > self.stall_s

    @property
    def ready(self) -> bool:
        if self._failed or not self._t.is_alive():
            return False
        st = self.stalled()
        if st != self._stall_logged:
            self._stall_logged = st
            if st:
                _log.error("engine loop stalled for more than %.0f s: not ready", self.stall_s)
            else:
                _log.warning("engine loop resumed")
        return not st

    def shutdown(self):
        self._stop = True
        self._wake.set()
        self._t.join(timeout=10)

    def _run(self):
        eng = self.engine
        while not self._stop:
            self._beat = time.monotonic()
            while True:
                try:
                    s = self._in.get_nowait()
                except queue.Empty:
                    break
                try:
                    kw = {"lora": s.lora} if s.lora else {}
                    if s.images:
                        kw["images"] = s.images
                    eng.add_request(s.prompt, s.params, request_id=s.rid, **kw)
                    self._subs[s.rid] = s
                    self.metrics.requests_started()
                except Exception as e:  # bad request: report and drop
                    _log.warning("request %d rejected: %s", s.rid, e)
                    s.loop.call_soon_threadsafe(s.q.put_nowait, ("error", str(e)))
            while True:
                try:
                    rid = self._abort.get_nowait()
                except queue.Empty:
                    break
                if rid in self._subs:
                    eng.abort(rid)
                    self._finish(rid, "aborted")
            while True:
                try:
                    fn, fut, loop = self._calls.get_nowait()
                except queue.Empty:
                    break
                try:
                    r = fn(eng)
                    loop.call_soon_threadsafe(lambda f=fut, v=r: f.done() or f.set_result(v))
                except Exception as e:
                    loop.call_soon_threadsafe(lambda f=fut, x=e: f.done() or f.set_exception(x))
            if not eng.has_work():
                self._wake.wait(0.05)
                self._wake.clear()
                continue
            try:
                t0 = time.perf_counter()
                self._step_since = time.monotonic()
                try:
                    outs = eng.step()
                finally:
                    self._step_since = None
                self.metrics.step(time.perf_counter() - t0, len(outs))
            except Exception as e:  # engine failure: fail every request in flight
                _log.exception("engine step failed; %d requests failed", len(self._subs))
                self._failed = True
                for rid in list(self._subs):
                    s = self._subs.pop(rid)
                    s.loop.call_soon_threadsafe(s.q.put_nowait, ("error", repr(e)))
                continue
            for rid, tok, fin in outs:
                s = self._subs.get(rid)
                if s is None:
                    continue
                if tok is None:  # the engine could not serve it (e.g. its replica failed)
                    err = getattr(eng, "error_of", lambda r: None)(rid) or "request failed"
                    self._subs.pop(rid, None)
                    try:
                        eng.release(rid)
                    except Exception:
                        pass
                    s.loop.call_soon_threadsafe(s.q.put_nowait, ("error", err))
                    continue
                s.loop.call_soon_threadsafe(s.q.put_nowait, ("token", tok))
                if fin:
                    self._finish(rid, "length")

    def _finish(self, rid: int, reason: str):
        s = self._subs.pop(rid, None)
        tr = self.engine.traces.pop(rid, None)
        if tr is not None:
            tr.finish(time.perf_counter())
            self.metrics.request_done(tr)
        try:
            self.engine.release(rid)
        except Exception:
            pass
        if s is not None:
            s.loop.call_soon_threadsafe(s.q.put_nowait, ("done", reason, tr))


class ApiError(Exception):
    def __init__(self, status: int, message: str, kind: str = "invalid_request_error"):
        super().__init__(message)
        self.status, self.message, self.kind = status, message, kind


@dataclass
class Result:
    """One finished generation."""
    text: str = ""
    calls: list = field(default_factory=list)
    finish: str = "stop"            # stop | length | tool_calls
    n_prompt: int = 0
    n_out: int = 0
    trace: object = None
    rest: str = ""                  # content not yet streamed when the result arrived


class Serving:
    """What every route shares: the engine, tokenizer, templates and the one
    generation path (tools, response_format, LoRA selection, stop strings)."""

    def __init__(self, aengine: AsyncEngine, tokenizer, model_name: str, arch: str = "llama",
                 chat_template: str | None = None, max_model_len: int = 4096):
        self.ae, self.tok, self.model_name = aengine, tokenizer, model_name
        self.arch, self.template, self.max_model_len = arch, chat_template, max_model_len
        self.eos = getattr(tokenizer, "eos_id", -1)
        self._pieces: dict[int, str] = {}
        self.started = time.time()

    # ---------------------------------------------------------------- request parsing
    def lora_of(self, body: dict) -> str | None:
        """The LoRA adapter a request's "model" names (None: the base model)."""
        names = getattr(self.ae.engine, "lora_names", None) or []
        m = body.get("model")
        if not m or not names or m == self.model_name:
            return None
        name = m.split(":", 1)[1] if ":" in m and m.split(":", 1)[0] == self.model_name else m
        if name in names:
            return name
        return None

    def models(self) -> list[str]:
        return [self.model_name] + [f"{self.model_name}:{n}" for n in
                                    getattr(self.ae.engine, "lora_names", None) or [] if n]

    def prompt_len(self, ids, images) -> int:
        """Positions the prompt takes once each image marker is its rows."""
        v = getattr(self.ae.engine, "vision", None)
        return len(ids) + (len(images) * (v.rows_per_image - 1) if images and v else 0)

    def params(self, body: dict, n_prompt: int, response_format: dict | None = None) -> SamplingParams:
        if body.get("logprobs") or body.get("top_logprobs"):
            # refused rather than ignored, so a client never reads a missing field as "none"
            # (reference behaviour: src/api/openai/mod.rs:298-311)
            raise ApiError(400, "logprobs are not returned by this server; remove `logprobs` "
                                "and `top_logprobs` from the request")
        mt = body.get("max_tokens", body.get("max_completion_tokens", body.get("max_output_tokens")))
        if mt is None:
            mt = max(1, min(1024, self.max_model_len - n_prompt))
        if int(mt) < 1:
            raise ApiError(400, "max_tokens must be at least 1")
        if n_prompt + int(mt) > self.max_model_len:
            raise ApiError(400, f"prompt ({n_prompt}) + max_tokens ({mt}) exceeds the "
                                f"context window ({self.max_model_len})")
        t = body.get("temperature")
        rf = response_format or body.get("response_format") or {}
        constraint = None
        if isinstance(rf, dict) and rf.get("type") in ("json_object", "json_schema"):
            from .json_guard import JsonConstraint
            schema = None
            if rf.get("type") == "json_schema":
                schema = (rf.get("json_schema") or {}).get("schema")
            constraint = JsonConstraint(self.piece, int(self.eos),
                                        schema=schema if isinstance(schema, dict) else None)
        bias = None
        lb = body.get("logit_bias")
        if lb:
            if not isinstance(lb, dict):
                raise ApiError(400, "logit_bias must map token ids to numbers")
            try:
                bias = {int(k): max(-100.0, min(100.0, float(v))) for k, v in lb.items()}
            except (TypeError, ValueError):
                raise ApiError(400, "logit_bias must map token ids to numbers")
        return SamplingParams(max_tokens=int(mt), temperature=float(1.0 if t is None else t),
                              constraint=constraint, logit_bias=bias,
                              top_p=float(body.get("top_p", 1.0) or 1.0),
                              top_k=int(body.get("top_k", 0) or 0),
                              seed=self.seed_of(body), eos_token_id=int(self.eos),
                              ignore_eos=bool(body.get("ignore_eos", False)),
                              frequency_penalty=float(body.get("frequency_penalty", 0.0) or 0.0),
                              presence_penalty=float(body.get("presence_penalty", 0.0) or 0.0))

    @staticmethod
    def seed_of(body: dict) -> int:
        """The client's seed, or a fresh random one: unseeded sampled requests
        must not all draw the same tokens for the same prompt."""
        seed = body.get("seed")
        if seed is None:
            return secrets.randbits(62)
        try:
            return int(seed)
        except (TypeError, ValueError):
            raise ApiError(400, "seed must be an integer")

    def piece(self, tok: int) -> str:
        """Text of one token (cached: the JSON constraint asks for many)."""
        p = self._pieces.get(tok)
        if p is None:
            p = self._pieces[tok] = self.tok.decode([tok])
        return p

    MAX_N = 16

    def n_of(self, body: dict) -> int:
        """How many independent choices a request asks for (OpenAI `n`)."""
        n = body.get("n", 1)
        if n is None:
            return 1
        if not isinstance(n, int) or isinstance(n, bool) or not 1 <= n <= self.MAX_N:
            raise ApiError(400, f"n must be an integer from 1 to {self.MAX_N}")
        if n > 1 and body.get("stream"):
            raise ApiError(400, "n > 1 is served without streaming only; set stream to false")
        return n

    @staticmethod
    def variants(sp: SamplingParams, n: int) -> list[SamplingParams]:
        """n request parameter sets: their own constraint state, and when
        sampling, consecutive seeds so the choices differ."""
        out = []
        for i in range(n):
            seed = sp.seed + i if sp.temperature > 0 else sp.seed
            c = sp.constraint.fresh() if (sp.constraint is not None and i) else sp.constraint
            out.append(dataclasses.replace(sp, seed=seed, constraint=c))
        return out

    @staticmethod
    def stops(body: dict) -> list[str]:
        st = body.get("stop") or body.get("stop_sequences") or []
        return [st] if isinstance(st, str) else list(st)

    def prepare(self, messages: list[dict], tools: list[ToolSpec] | None = None, tool_choice=None,
                response_format: dict | None = None) -> tuple[list[int], list[ToolSpec], list]:
        """Token ids of the rendered conversation (IMAGE_TOKEN where an image
        goes), the tools that stay active, and the images (encoded bytes)."""
        images: list = []
        msgs = [self._flatten(m, images) for m in messages]
        extra = []
        if tools and not tool_choice_forbids(tool_choice):
            extra.append(format_tool_prompt(tools, tool_choice))
        else:
            tools = []
        if response_format and response_format.get("type") in ("json_object", "json_schema"):
            s = "Reply with one valid JSON object and nothing else."
            schema = (response_format.get("json_schema") or {}).get("schema")
            if schema:
                s += " It must conform to this JSON schema: " + json.dumps(schema)
            extra.append(s)
        if extra:
            text = "\n\n".join(extra)
            if msgs and msgs[0]["role"] == "system":
                msgs[0] = {"role": "system", "content": msgs[0]["content"] + "\n\n" + text}
            else:
                msgs.insert(0, {"role": "system", "content": text})
        text = render(msgs, self.arch, self.template)
        if not images:
            return self.tok.encode(text), tools, images
        if getattr(self.ae.engine, "vision", None) is None:
            raise ApiError(400, "this model takes no image input (start the server with --mmproj)")
        from ..models.vision import IMAGE_TOKEN, MEDIA_MARKER
        pieces = text.split(MEDIA_MARKER)
        ids = self.tok.encode(pieces[0])
        for piece in pieces[1:]:
            ids.append(IMAGE_TOKEN)
            ids += self.tok.encode(piece, add_bos=False)
        return ids, tools, images

    @staticmethod
    def _flatten(m: dict, images: list | None = None) -> dict:
        """One message with plain-text content: assistant tool calls become the
        JSON shape the tool prompt asks for; tool results become text; images
        (inline data only) become a marker, their bytes appended to `images`."""
        role = m.get("role", "user")
        c = m.get("content", "")
        if isinstance(c, list):
            parts = []
            for p in c:
                if not isinstance(p, dict):
                    continue
                t = p.get("type")
                if t in ("image_url", "image", "input_image"):
                    from ..models.vision import MEDIA_MARKER
                    if images is None:
                        raise ApiError(400, "images are not accepted here")
                    images.append(_image_bytes(p))
                    parts.append(MEDIA_MARKER)
                elif t in ("text", "input_text", "output_text"):
                    parts.append(p.get("text", ""))
                elif t == "tool_use":
                    parts.append(json.dumps({"tool_calls": [{"name": p.get("name"),
                                                             "arguments": p.get("input", {})}]}))
                elif t == "tool_result":
                    inner = p.get("content", "")
                    if isinstance(inner, list):
                        inner = "".join(x.get("text", "") for x in inner if isinstance(x, dict))
                    parts.append(f"[tool result {p.get('tool_use_id', '')}] {inner}")
            c = "".join(parts)
        calls = m.get("tool_calls")
        if calls:
            c = (c or "") + json.dumps({"tool_calls": [
                {"name": (x.get("function") or x).get("name"),
                 "arguments": _loads_or((x.get("function") or x).get("arguments"))} for x in calls]})
        if role == "tool":
            c = f"[tool result {m.get('tool_call_id', '')}] {c}"
        return {"role": role, "content": c or ""}

    # ---------------------------------------------------------------- generation
    async def stream(self, ids, sp: SamplingParams, stops: list[str], tools=None,
                     lora: str | None = None, images=None):
        """Async generator of events:
             ("text", delta)          content to show now
             ("done", Result)         at the end (calls parsed, counts, trace)."""
        rid, q = self.ae.submit(ids, sp, lora, images)
        toks: list[int] = []
        text = ""
        sent = 0
        try:
            while True:
                msg = await q.get()
                if msg[0] == "error":
                    raise ApiError(500, msg[1], "server_error")
                if msg[0] == "done":
                    fin = "length" if len(toks) >= sp.max_tokens else "stop"
                    yield self._finish(text, sent, tools, fin, self.prompt_len(ids, images), len(toks),
                                       msg[2])
                    return
                toks.append(msg[1])
                if msg[1] == self.eos and not sp.ignore_eos:
                    continue
                text = self.tok.decode([t for t in toks if t != self.eos or sp.ignore_eos])
                hit = min((text.index(s) for s in stops if s in text), default=-1)
                if hit >= 0:
                    text = text[:hit]
                    self.ae.abort(rid)
                    yield self._finish(text, sent, tools, "stop", self.prompt_len(ids, images),
                                       len(toks), None)
                    return
                safe = content_prefix_len(text) if tools else len(text)
                if safe > sent:
                    yield ("text", text[sent:safe])
                    sent = safe
        except asyncio.CancelledError:
            self.ae.abort(rid)
            raise

    @staticmethod
    def _finish(text, sent, tools, fin, n_prompt, n_out, trace):
        r = Result(text=text, finish=fin, n_prompt=n_prompt, n_out=n_out, trace=trace)
        parsed = parse_tool_calls(text, tools) if tools else None
        if parsed is not None:
            r.text, r.calls, r.finish = parsed[0], parsed[1], "tool_calls"
        r.rest = r.text[sent:] if len(r.text) > sent else ""
        return ("done", r)

    async def run(self, ids, sp, stops, tools=None, lora=None, images=None) -> Result:
        async for ev in self.stream(ids, sp, stops, tools, lora, images):
            if ev[0] == "done":
                return ev[1]
        raise ApiError(500, "generation ended without a result", "server_error")


def _image_bytes(part: dict) -> bytes:
    """Encoded image bytes of an OpenAI (image_url / input_image data URL) or
    Anthropic (base64 source) content part.  No fetching: inline data only."""
    import base64
    src = part.get("source")
    if isinstance(src, dict):                      # Anthropic
        if src.get("type") != "base64":
            raise ApiError(400, "only base64 image sources are accepted")
        data = src.get("data", "")
    else:
        url = part.get("image_url")
        url = url.get("url") if isinstance(url, dict) else url
        if not isinstance(url, str) or not url.startswith("data:") or "," not in url:
            raise ApiError(400, "images must be data: URLs (this server fetches nothing)")
        data = url.split(",", 1)[1]
    try:
        return base64.b64decode(data, validate=False)
    except ValueError:
        raise ApiError(400, "image data is not base64")


def _loads_or(v):
    if isinstance(v, str):
        try:
            return json.loads(v)
        except ValueError:
            return v
    return v if v is not None else {}


def create_app(aengine: AsyncEngine, tokenizer, model_name: str, arch: str = "llama",
               chat_template: str | None = None, max_model_len: int = 4096,
               api_key: str | None = None, cors_origins=(), rpm: int = 0, port: int = 8800,
               store_path: str | None = None, config_path: str | None = None,
               api_key_file: str | None = None):
    """`api_key_file`: the key is read from it when `api_key` is not given,
    and a key rotated through the admin API is written back to it."""
    from fastapi import FastAPI
    from fastapi.responses import JSONResponse, PlainTextResponse, StreamingResponse

    from . import admin, mcp, responses
    from .middleware import SecurityMiddleware, ServerSettings

    app = FastAPI(title="swarmllm_b200")
    S = Serving(aengine, tokenizer, model_name, arch, chat_template, max_model_len)
    app.state.serving = S

    @app.exception_handler(ApiError)
    async def _api_error(request: Request, e: ApiError):
        if request.url.path.startswith("/v1/messages"):
            return JSONResponse({"type": "error", "error": {"type": e.kind, "message": e.message}},
                                status_code=e.status)
        return JSONResponse({"error": {"message": e.message, "type": e.kind}}, status_code=e.status)

    def headers_of(tr) -> dict:
        return tr.headers() if tr is not None else {}

    async def body_of(request: Request) -> dict:
        try:
            body = await request.json()
        except ValueError:
            raise ApiError(400, "request body is not valid JSON")
        if not isinstance(body, dict):
            raise ApiError(400, "request body must be a JSON object")
        return body

    def sse(obj) -> str:
        return f"data: {json.dumps(obj)}\n\n"

    # ------------------------------------------------------------------ OpenAI chat
    @app.post("/v1/chat/completions")
    async def chat_completions(request: Request):
        body = await body_of(request)
        msgs = body.get("messages")
        if not msgs:
            raise ApiError(400, "messages is required")
        try:
            tools = tools_from_openai(body.get("tools"))
        except ValueError as e:
            raise ApiError(400, str(e))
        ids, tools, images = S.prepare(msgs, tools, body.get("tool_choice"), body.get("response_format"))
        sp = S.params(body, S.prompt_len(ids, images))
        n = S.n_of(body)
        lora = S.lora_of(body)
        stops = S.stops(body)
        cid = "chatcmpl-" + uuid.uuid4().hex[:24]
        created = int(time.time())
        model = body.get("model") or model_name

        def chunk(delta, fin=None):
            return sse({"id": cid, "object": "chat.completion.chunk", "created": created,
                        "model": model, "choices": [{"index": 0, "delta": delta, "finish_reason": fin}]})

        if body.get("stream"):
            async def gen():
                yield chunk({"role": "assistant"})
                async for ev in S.stream(ids, sp, stops, tools, lora, images):
                    if ev[0] == "text":
                        yield chunk({"content": ev[1]})
                        continue
                    r = ev[1]
                    if r.rest:
                        yield chunk({"content": r.rest})
                    if r.calls:
                        yield chunk({"tool_calls": [dict(c.openai(), index=i)
                                                    for i, c in enumerate(r.calls)]})
                    yield chunk({}, r.finish)
                    if (body.get("stream_options") or {}).get("include_usage"):
                        yield sse({"id": cid, "object": "chat.completion.chunk", "created": created,
                                   "model": model, "choices": [],
                                   "usage": {"prompt_tokens": r.n_prompt, "completion_tokens": r.n_out,
                                             "total_tokens": r.n_prompt + r.n_out}})
                yield "data: [DONE]\n\n"
            return StreamingResponse(gen(), media_type="text/event-stream")
        rs = await asyncio.gather(*[S.run(ids, v, stops, tools, lora, images)
                                    for v in S.variants(sp, n)])
        choices = []
        for i, r in enumerate(rs):
            msg = {"role": "assistant", "content": r.text if (r.text or not r.calls) else None}
            if r.calls:
                msg["tool_calls"] = [c.openai() for c in r.calls]
            choices.append({"index": i, "message": msg, "finish_reason": r.finish})
        n_out = sum(r.n_out for r in rs)
        return JSONResponse({
            "id": cid, "object": "chat.completion", "created": created, "model": model,
            "choices": choices,
            "usage": {"prompt_tokens": rs[0].n_prompt, "completion_tokens": n_out,
                      "total_tokens": rs[0].n_prompt + n_out}}, headers=headers_of(rs[0].trace))

    # ------------------------------------------------------------------ OpenAI completions
    @app.post("/v1/completions")
    async def completions(request: Request):
        body = await body_of(request)
        p = body.get("prompt", "")
        # OpenAI prompt forms: a string, a token-id list, or a batch of either
        # (each batch entry gets its own n choices, indexed prompt-major).
        if isinstance(p, list) and p and all(isinstance(x, int) for x in p):
            batch = [list(p)]
        elif isinstance(p, list) and p and all(isinstance(x, (str, list)) for x in p):
            batch = [list(x) if isinstance(x, list) else tokenizer.encode(x) for x in p]
            if not all(all(isinstance(t, int) for t in b) for b in batch):
                raise ApiError(400, "prompt lists must hold strings or token-id lists")
        elif isinstance(p, str):
            batch = [tokenizer.encode(p)]
        else:
            raise ApiError(400, "prompt must be a string, a token-id list, or a list of those")
        n = S.n_of(body)
        lora = S.lora_of(body)
        cid = "cmpl-" + uuid.uuid4().hex[:24]
        echo = bool(body.get("echo"))

        def head_of(ids):  # echo: the prompt text ahead of each completion
            return tokenizer.decode([t for t in ids if t != S.eos]) if echo else ""
        if body.get("stream"):
            if len(batch) != 1:
                raise ApiError(400, "streaming serves one prompt per request")
            ids = batch[0]
            sp = S.params(body, len(ids))

            async def gen():
                if echo:
                    yield sse({"id": cid, "object": "text_completion", "model": model_name,
                               "choices": [{"index": 0, "text": head_of(ids), "finish_reason": None}]})
                async for ev in S.stream(ids, sp, S.stops(body), None, lora):
                    if ev[0] == "text":
                        ch = {"id": cid, "object": "text_completion", "model": model_name,
                              "choices": [{"index": 0, "text": ev[1], "finish_reason": None}]}
                    else:
                        ch = {"id": cid, "object": "text_completion", "model": model_name,
                              "choices": [{"index": 0, "text": ev[1].rest, "finish_reason": ev[1].finish}]}
                    yield sse(ch)
                yield "data: [DONE]\n\n"
            return StreamingResponse(gen(), media_type="text/event-stream")
        if len(batch) * n > S.MAX_N:
            raise ApiError(400, f"at most {S.MAX_N} completions (prompts x n) per request")
        jobs = []
        for ids in batch:
            sp = S.params(body, len(ids))
            jobs += [(ids, v) for v in S.variants(sp, n)]
        rs = await asyncio.gather(*[S.run(ids, v, S.stops(body), None, lora) for ids, v in jobs])
        n_out = sum(r.n_out for r in rs)
        n_prompt = sum(rs[i * n].n_prompt for i in range(len(batch)))
        return {"id": cid, "object": "text_completion", "model": model_name,
                "choices": [{"index": i, "text": head_of(ids) + r.text, "finish_reason": r.finish}
                            for i, ((ids, _), r) in enumerate(zip(jobs, rs))],
                "usage": {"prompt_tokens": n_prompt, "completion_tokens": n_out,
                          "total_tokens": n_prompt + n_out}}

    # ------------------------------------------------------------------ Anthropic messages
    @app.post("/v1/messages")
    async def messages(request: Request):
        body = await body_of(request)
        msgs = list(body.get("messages") or [])
        if not msgs:
            raise ApiError(400, "messages is required")
        sysmsg = body.get("system")
        if sysmsg:
            msgs = [{"role": "system", "content": sysmsg if isinstance(sysmsg, str) else
                     "".join(b.get("text", "") for b in sysmsg)}] + msgs
        ids, tools, images = S.prepare(msgs, tools_from_anthropic(body.get("tools")), body.get("tool_choice"))
        sp = S.params(body, S.prompt_len(ids, images))
        lora = S.lora_of(body)
        mid = "msg_" + uuid.uuid4().hex[:24]
        stop_of = {"length": "max_tokens", "tool_calls": "tool_use", "stop": "end_turn"}
        if body.get("stream"):
            async def gen():
                def ev(kind, data):
                    return f"event: {kind}\ndata: {json.dumps(data)}\n\n"
                yield ev("message_start", {"type": "message_start", "message": {
                    "id": mid, "type": "message", "role": "assistant", "model": body.get("model", model_name),
                    "content": [], "stop_reason": None,
                    "usage": {"input_tokens": len(ids), "output_tokens": 0}}})
                opened = False
                async for e in S.stream(ids, sp, S.stops(body), tools, lora, images):
                    delta = e[1] if e[0] == "text" else e[1].rest
                    if delta:
                        if not opened:
                            yield ev("content_block_start", {"type": "content_block_start", "index": 0,
                                                             "content_block": {"type": "text", "text": ""}})
                            opened = True
                        yield ev("content_block_delta", {"type": "content_block_delta", "index": 0,
                                                         "delta": {"type": "text_delta", "text": delta}})
                    if e[0] != "done":
                        continue
                    r = e[1]
                    idx = 0
                    if opened:
                        yield ev("content_block_stop", {"type": "content_block_stop", "index": 0})
                        idx = 1
                    for c in r.calls:
                        blk = c.anthropic()
                        yield ev("content_block_start", {"type": "content_block_start", "index": idx,
                                                         "content_block": dict(blk, input={})})
                        yield ev("content_block_delta", {"type": "content_block_delta", "index": idx,
                                                         "delta": {"type": "input_json_delta",
                                                                   "partial_json": c.arguments}})
                        yield ev("content_block_stop", {"type": "content_block_stop", "index": idx})
                        idx += 1
                    yield ev("message_delta", {"type": "message_delta",
                                               "delta": {"stop_reason": stop_of[r.finish], "stop_sequence": None},
                                               "usage": {"output_tokens": r.n_out}})
                yield ev("message_stop", {"type": "message_stop"})
            return StreamingResponse(gen(), media_type="text/event-stream")
        r = await S.run(ids, sp, S.stops(body), tools, lora, images)
        content = ([{"type": "text", "text": r.text}] if r.text or not r.calls else []) + \
            [c.anthropic() for c in r.calls]
        return {"id": mid, "type": "message", "role": "assistant", "model": body.get("model", model_name),
                "content": content, "stop_reason": stop_of[r.finish], "stop_sequence": None,
                "usage": {"input_tokens": r.n_prompt, "output_tokens": r.n_out}}

    # ------------------------------------------------------------------ embeddings
    @app.post("/v1/embeddings")
    async def embeddings(request: Request):
        body = await body_of(request)
        inp = body.get("input", "")
        texts = [inp] if isinstance(inp, str) else list(inp)
        out = []
        for i, t in enumerate(texts):
            ids = list(t) if isinstance(t, list) else tokenizer.encode(t, add_bos=False)
            vec = aengine.engine.embed_text(ids)
            out.append({"object": "embedding", "index": i, "embedding": vec})
        return {"object": "list", "data": out, "model": model_name}

    # ------------------------------------------------------------------ info / health / metrics
    @app.get("/v1/models")
    async def models():
        return {"object": "list", "data": [{"id": m, "object": "model", "owned_by": "local",
                                            "max_model_len": max_model_len} for m in S.models()]}

    @app.get("/v1/models/{mid:path}")
    async def model_one(mid: str):
        if mid not in S.models() and S.lora_of({"model": mid}) is None:
            raise ApiError(404, f"The model '{mid}' does not exist")
        return {"id": mid, "object": "model", "owned_by": "local", "max_model_len": max_model_len}

    @app.post("/v1/messages/count_tokens")
    async def count_tokens(request: Request):
        """Anthropic token count of a messages request (system, tools and images included)."""
        body = await body_of(request)
        msgs = list(body.get("messages") or [])
        if not msgs:
            raise ApiError(400, "messages is required")
        sysmsg = body.get("system")
        if sysmsg:
            msgs = [{"role": "system", "content": sysmsg if isinstance(sysmsg, str) else
                     "".join(b.get("text", "") for b in sysmsg)}] + msgs
        ids, _, images = S.prepare(msgs, tools_from_anthropic(body.get("tools")), body.get("tool_choice"))
        return {"input_tokens": S.prompt_len(ids, images)}

    @app.get("/health")
    async def health():
        return {"status": "ok"}

    @app.get("/health/ready")
    async def ready():
        if not aengine.ready:
            return JSONResponse({"status": "unavailable"}, status_code=503)
        return {"status": "ready"}

    def status_dict() -> dict:
        e = aengine.engine
        return {"model": model_name, "models": S.models(), "running": e.sched.num_running,
                "waiting": e.sched.num_waiting, "kv_pages_free": e.bm.num_free(),
                "kv_pages": e.bm.num_pages, "prefix_cache_hit_tokens": e.bm.prefix_hit_tokens,
                "steps": e.steps, "uptime_s": round(time.time() - S.started, 1),
                "ready": aengine.ready}
    S.status = status_dict

    @app.get("/api/status")
    async def status():
        return status_dict()

    @app.get("/v1/status")
    async def v1_status():
        return status_dict()

    @app.get("/metrics")
    async def metrics():
        e = aengine.engine
        aengine.metrics.set_kv(e.bm.num_free(), e.bm.num_pages)
        aengine.metrics.set_engine(e, aengine.ready)
        return PlainTextResponse(aengine.metrics.render(), media_type="text/plain; version=0.0.4")

    # ------------------------------------------------------------------ prefix KV snapshots
    @app.post("/api/prefix/export")
    async def prefix_export(request: Request):
        """Body {"prompt": text} or {"tokens": [...]}: the cached KV pages of that
        prefix as a snapshot (application/octet-stream; 204 if none cached)."""
        from fastapi.responses import Response
        body = await body_of(request)
        toks = body.get("tokens")
        if toks is None:
            toks = tokenizer.encode(body.get("prompt", ""))
        snap = await aengine.call(lambda e: e.export_prefix(list(toks)))
        if snap is None:
            return Response(status_code=204)
        return Response(snap.to_bytes(), media_type="application/octet-stream",
                        headers={"x-swarmllm-prefix-tokens": str(len(snap.tokens))})

    @app.post("/api/prefix/import")
    async def prefix_import(request: Request):
        from ..engine.prefix_share import PrefixSnapshot
        raw = await request.body()
        try:
            snap = PrefixSnapshot.from_bytes(raw)
        except (ValueError, KeyError) as e:
            raise ApiError(400, f"bad snapshot: {e}")
        try:
            n = await aengine.call(lambda e: e.import_prefix(snap))
        except (ValueError, RuntimeError) as e:
            raise ApiError(400, str(e))
        return {"imported_tokens": n, "snapshot_tokens": len(snap.tokens)}

    @app.websocket("/api/admin/ws")
    async def ws_feed(ws: WebSocket):
        """Dashboard feed: the status dict once a second until the client leaves."""
        await ws.accept()
        try:
            n = int(ws.query_params.get("n", "0") or 0)   # n > 0: stop after n messages
            i = 0
            while True:
                await ws.send_json(dict(status_dict(), type="status", seq=i))
                i += 1
                if n and i >= n:
                    break
                await asyncio.sleep(1.0)
        except Exception:
            pass
        finally:
            try:
                await ws.close()
            except Exception:
                pass

    if not api_key and api_key_file and os.path.exists(api_key_file):
        with open(api_key_file) as f:
            api_key = f.read().strip() or None
    settings = ServerSettings(api_key or None, port, tuple(cors_origins), rpm,
                              key_file=api_key_file)
    app.state.settings = settings
    responses.register(app, S, store_path)
    mcp.register(app, S)
    admin.register(app, S, settings, config_path)
    app.add_middleware(SecurityMiddleware, settings=settings)
    return app


def serve(engine, tokenizer, model_name: str, host: str = "0.0.0.0", port: int = 8800, **kw):
    import uvicorn
    ae = AsyncEngine(engine)
    app = create_app(ae, tokenizer, model_name, port=port, **kw)
    server = uvicorn.Server(uvicorn.Config(app, host=host, port=port, log_level="info"))
    app.state.shutdown_hook = lambda: setattr(server, "should_exit", True)   # admin shutdown
    try:
        server.run()
    finally:
        ae.shutdown()
