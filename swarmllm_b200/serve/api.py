"""OpenAI- and Anthropic-compatible HTTP API on port 8800.

Routes (reference: src/api/server.rs:239-559, src/api/openai/mod.rs:319,
src/api/openai/streaming.rs:1431, src/api/anthropic/):
  POST /v1/chat/completions    (stream=true -> SSE chunks, data: [DONE])
  POST /v1/completions
  POST /v1/messages            (Anthropic Messages; stream -> typed SSE events)
  POST /v1/embeddings          (mean-pooled, L2-normalised input embeddings)
  GET  /v1/models
  GET  /health, /health/ready, /metrics (Prometheus), /api/status

The engine is single-threaded: ``AsyncEngine`` runs ``step()`` in a worker
thread, takes new requests from a queue between steps and hands each token
to the request's asyncio queue.  Continuous batching therefore happens
across HTTP requests automatically.
"""
from __future__ import annotations

import asyncio
import itertools
import json
import queue
import threading
import time
import uuid
from dataclasses import dataclass

from fastapi import Request  # module level: route annotations are resolved from globals

from ..engine.sampling import SamplingParams
from ..utils.metrics import Metrics
from .chat_template import render


@dataclass
class _Sub:
    rid: int
    prompt: list
    params: SamplingParams
    q: asyncio.Queue
    loop: asyncio.AbstractEventLoop


class AsyncEngine:
    def __init__(self, engine, metrics: Metrics | None = None):
        self.engine = engine
        self.metrics = metrics or Metrics()
        self._in: queue.Queue = queue.Queue()
        self._abort: queue.Queue = queue.Queue()
        self._subs: dict[int, _Sub] = {}
        self._ids = itertools.count(1)
        self._wake = threading.Event()
        self._stop = False
        self.ready = True
        self._t = threading.Thread(target=self._run, daemon=True, name="engine")
        self._t.start()

    def submit(self, prompt_ids, params: SamplingParams) -> tuple[int, asyncio.Queue]:
        rid = next(self._ids)
        q: asyncio.Queue = asyncio.Queue()
        self._in.put(_Sub(rid, list(prompt_ids), params, q, asyncio.get_running_loop()))
        self._wake.set()
        return rid, q

    def abort(self, rid: int):
        self._abort.put(rid)
        self._wake.set()

    def shutdown(self):
        self._stop = True
        self._wake.set()
        self._t.join(timeout=10)

    def _run(self):
        eng = self.engine
        while not self._stop:
            while True:
                try:
                    s = self._in.get_nowait()
                except queue.Empty:
                    break
                try:
                    eng.add_request(s.prompt, s.params, request_id=s.rid)
                    self._subs[s.rid] = s
                    self.metrics.requests_started()
                except Exception as e:  # bad request: report and drop
                    s.loop.call_soon_threadsafe(s.q.put_nowait, ("error", str(e)))
            while True:
                try:
                    rid = self._abort.get_nowait()
                except queue.Empty:
                    break
                if rid in self._subs:
                    eng.abort(rid)
                    self._finish(rid, "aborted")
            if not eng.has_work():
                self._wake.wait(0.05)
                self._wake.clear()
                continue
            try:
                t0 = time.perf_counter()
                outs = eng.step()
                self.metrics.step(time.perf_counter() - t0, len(outs))
            except Exception as e:  # engine failure: fail every request in flight
                self.ready = False
                for rid in list(self._subs):
                    s = self._subs.pop(rid)
                    s.loop.call_soon_threadsafe(s.q.put_nowait, ("error", repr(e)))
                continue
            for rid, tok, fin in outs:
                s = self._subs.get(rid)
                if s is None:
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


def create_app(aengine: AsyncEngine, tokenizer, model_name: str, arch: str = "llama",
               chat_template: str | None = None, max_model_len: int = 4096):
    from fastapi import FastAPI, HTTPException
    from fastapi.responses import JSONResponse, PlainTextResponse, StreamingResponse

    app = FastAPI(title="swarmllm_b200")
    eos = getattr(tokenizer, "eos_id", -1)

    def params_from(body: dict, n_prompt: int) -> SamplingParams:
        mt = body.get("max_tokens", body.get("max_completion_tokens"))
        if mt is None:
            mt = max(1, min(1024, max_model_len - n_prompt))
        if n_prompt + int(mt) > max_model_len:
            raise HTTPException(400, f"prompt ({n_prompt}) + max_tokens ({mt}) exceeds the "
                                     f"context window ({max_model_len})")
        return SamplingParams(max_tokens=int(mt), temperature=float(body.get("temperature", 1.0)),
                              top_p=float(body.get("top_p", 1.0)), top_k=int(body.get("top_k", 0) or 0),
                              seed=int(body.get("seed", 0) or 0), eos_token_id=int(eos),
                              ignore_eos=bool(body.get("ignore_eos", False)))

    def stops_of(body: dict) -> list[str]:
        st = body.get("stop") or body.get("stop_sequences") or []
        return [st] if isinstance(st, str) else list(st)

    async def generate(prompt_ids, sp: SamplingParams, stops: list[str]):
        """Async generator of (text_delta, finish_reason|None, trace|None)."""
        rid, q = aengine.submit(prompt_ids, sp)
        toks: list[int] = []
        emitted = ""
        try:
            while True:
                msg = await q.get()
                if msg[0] == "error":
                    raise HTTPException(500, msg[1])
                if msg[0] == "done":
                    yield "", ("length" if len(toks) >= sp.max_tokens else "stop"), msg[2]
                    return
                toks.append(msg[1])
                if msg[1] == eos and not sp.ignore_eos:
                    continue
                text = tokenizer.decode(toks)
                hit = next((s for s in stops if s in text), None)
                if hit is not None:
                    text = text[:text.index(hit)]
                    delta = text[len(emitted):]
                    emitted = text
                    aengine.abort(rid)
                    yield delta, "stop", None
                    return
                delta = text[len(emitted):]
                emitted = text
                if delta:
                    yield delta, None, None
        except asyncio.CancelledError:
            aengine.abort(rid)
            raise

    def headers_of(tr) -> dict:
        return tr.headers() if tr is not None else {}

    # ------------------------------------------------------------------ OpenAI chat
    @app.post("/v1/chat/completions")
    async def chat_completions(request: Request):
        body = await request.json()
        msgs = body.get("messages")
        if not msgs:
            raise HTTPException(400, "messages is required")
        prompt = render(msgs, arch, chat_template)
        ids = tokenizer.encode(prompt)
        sp = params_from(body, len(ids))
        stops = stops_of(body)
        cid = "chatcmpl-" + uuid.uuid4().hex[:24]
        created = int(time.time())
        if body.get("stream"):
            async def sse():
                first = {"id": cid, "object": "chat.completion.chunk", "created": created,
                         "model": model_name,
                         "choices": [{"index": 0, "delta": {"role": "assistant"}, "finish_reason": None}]}
                yield f"data: {json.dumps(first)}\n\n"
                n = 0
                async for delta, fin, tr in generate(ids, sp, stops):
                    if delta:
                        n += 1
                        ch = {"id": cid, "object": "chat.completion.chunk", "created": created,
                              "model": model_name,
                              "choices": [{"index": 0, "delta": {"content": delta}, "finish_reason": None}]}
                        yield f"data: {json.dumps(ch)}\n\n"
                    if fin:
                        end = {"id": cid, "object": "chat.completion.chunk", "created": created,
                               "model": model_name,
                               "choices": [{"index": 0, "delta": {}, "finish_reason": fin}]}
                        yield f"data: {json.dumps(end)}\n\n"
                yield "data: [DONE]\n\n"
            return StreamingResponse(sse(), media_type="text/event-stream")
        text, fin, trace = "", "stop", None
        async for delta, f, tr in generate(ids, sp, stops):
            text += delta
            if f:
                fin, trace = f, tr
        n_out = len(tokenizer.encode(text, add_bos=False)) if text else 0
        return JSONResponse({
            "id": cid, "object": "chat.completion", "created": created, "model": model_name,
            "choices": [{"index": 0, "message": {"role": "assistant", "content": text},
                         "finish_reason": fin}],
            "usage": {"prompt_tokens": len(ids), "completion_tokens": n_out,
                      "total_tokens": len(ids) + n_out}}, headers=headers_of(trace))

    # ------------------------------------------------------------------ OpenAI completions
    @app.post("/v1/completions")
    async def completions(request: Request):
        body = await request.json()
        p = body.get("prompt", "")
        ids = list(p) if isinstance(p, list) and p and isinstance(p[0], int) else tokenizer.encode(
            p if isinstance(p, str) else "".join(p))
        sp = params_from(body, len(ids))
        cid = "cmpl-" + uuid.uuid4().hex[:24]
        if body.get("stream"):
            async def sse():
                async for delta, fin, tr in generate(ids, sp, stops_of(body)):
                    ch = {"id": cid, "object": "text_completion", "model": model_name,
                          "choices": [{"index": 0, "text": delta, "finish_reason": fin}]}
                    yield f"data: {json.dumps(ch)}\n\n"
                yield "data: [DONE]\n\n"
            return StreamingResponse(sse(), media_type="text/event-stream")
        text, fin = "", "stop"
        async for delta, f, tr in generate(ids, sp, stops_of(body)):
            text += delta
            fin = f or fin
        return {"id": cid, "object": "text_completion", "model": model_name,
                "choices": [{"index": 0, "text": text, "finish_reason": fin}],
                "usage": {"prompt_tokens": len(ids)}}

    # ------------------------------------------------------------------ Anthropic messages
    @app.post("/v1/messages")
    async def messages(request: Request):
        body = await request.json()
        msgs = list(body.get("messages") or [])
        sysmsg = body.get("system")
        if sysmsg:
            msgs = [{"role": "system", "content": sysmsg if isinstance(sysmsg, str) else
                     "".join(b.get("text", "") for b in sysmsg)}] + msgs
        ids = tokenizer.encode(render(msgs, arch, chat_template))
        sp = params_from(body, len(ids))
        mid = "msg_" + uuid.uuid4().hex[:24]
        if body.get("stream"):
            async def sse():
                def ev(kind, data):
                    return f"event: {kind}\ndata: {json.dumps(data)}\n\n"
                yield ev("message_start", {"type": "message_start", "message": {
                    "id": mid, "type": "message", "role": "assistant", "model": model_name,
                    "content": [], "usage": {"input_tokens": len(ids), "output_tokens": 0}}})
                yield ev("content_block_start", {"type": "content_block_start", "index": 0,
                                                 "content_block": {"type": "text", "text": ""}})
                stop = "end_turn"
                async for delta, fin, tr in generate(ids, sp, stops_of(body)):
                    if delta:
                        yield ev("content_block_delta", {"type": "content_block_delta", "index": 0,
                                                         "delta": {"type": "text_delta", "text": delta}})
                    if fin == "length":
                        stop = "max_tokens"
                yield ev("content_block_stop", {"type": "content_block_stop", "index": 0})
                yield ev("message_delta", {"type": "message_delta", "delta": {"stop_reason": stop}})
                yield ev("message_stop", {"type": "message_stop"})
            return StreamingResponse(sse(), media_type="text/event-stream")
        text, stop = "", "end_turn"
        async for delta, f, tr in generate(ids, sp, stops_of(body)):
            text += delta
            if f == "length":
                stop = "max_tokens"
        return {"id": mid, "type": "message", "role": "assistant", "model": model_name,
                "content": [{"type": "text", "text": text}], "stop_reason": stop,
                "usage": {"input_tokens": len(ids)}}

    # ------------------------------------------------------------------ embeddings
    @app.post("/v1/embeddings")
    async def embeddings(request: Request):
        body = await request.json()
        inp = body.get("input", "")
        texts = [inp] if isinstance(inp, str) else list(inp)
        out = []
        for i, t in enumerate(texts):
            vec = aengine.engine.embed_text(tokenizer.encode(t, add_bos=False))
            out.append({"object": "embedding", "index": i, "embedding": vec})
        return {"object": "list", "data": out, "model": model_name}

    # ------------------------------------------------------------------ info / health / metrics
    @app.get("/v1/models")
    async def models():
        return {"object": "list", "data": [{"id": model_name, "object": "model", "owned_by": "local",
                                            "max_model_len": max_model_len}]}

    @app.get("/health")
    async def health():
        return {"status": "ok"}

    @app.get("/health/ready")
    async def ready():
        if not aengine.ready:
            return JSONResponse({"status": "unavailable"}, status_code=503)
        return {"status": "ready"}

    @app.get("/api/status")
    async def status():
        e = aengine.engine
        return {"model": model_name, "running": e.sched.num_running, "waiting": e.sched.num_waiting,
                "kv_pages_free": e.bm.num_free(), "kv_pages": e.bm.num_pages,
                "prefix_cache_hit_tokens": e.bm.prefix_hit_tokens, "steps": e.steps}

    @app.get("/metrics")
    async def metrics():
        e = aengine.engine
        aengine.metrics.set_kv(e.bm.num_free(), e.bm.num_pages)
        return PlainTextResponse(aengine.metrics.render(), media_type="text/plain; version=0.0.4")

    return app


def serve(engine, tokenizer, model_name: str, host: str = "0.0.0.0", port: int = 8800, **kw):
    import uvicorn
    ae = AsyncEngine(engine)
    app = create_app(ae, tokenizer, model_name, **kw)
    try:
        uvicorn.run(app, host=host, port=port, log_level="info")
    finally:
        ae.shutdown()
