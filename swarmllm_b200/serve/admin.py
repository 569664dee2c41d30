"""Admin API: the node's operational views and run-time controls.

  GET  /api/admin/stats          totals and last-minute rates (tok/s, busy
                                 fraction, step time, TTFT p50/p99)
  GET  /api/admin/performance    the same over 10 s / 60 s / 300 s windows
  GET  /api/admin/config         engine configuration and guard settings
  PUT  /api/admin/config         change guard settings (rpm, cors_origins,
                                 max_body) at run time
  POST /api/admin/config/reload  re-read the TOML config file given at start-up
                                 and apply its guard settings
  GET  /api/admin/models         the served model: architecture, size, weight
                                 types, LoRA adapters, image encoder
  POST /api/admin/lora           load a LoRA adapter GGUF ({"name", "path"})
  GET  /api/admin/diagnostics    devices (memory, SMs, clocks), software
                                 versions, native extensions loaded, KV cache
  GET  /api/admin/responses      stored /v1/responses ids (newest first)
  GET  /api/admin/storage        the model's files and their sizes (also /storage/breakdown)
  GET  /api/admin/adapters       LoRA adapters and their slots; POST loads one
  DELETE /api/admin/adapters/{id}  unload one (409 while a request uses it)
  GET  /api/admin/models/{id}    one served model (base or adapter); /status: loaded, ready
  GET  /api/admin/version        package and library versions
  GET  /api/admin/peers          none on one node (the GPUs are ranks, not peers)
  GET  /api/admin/schedule       scheduler state: running, waiting, preemptions, limits
  GET  /api/admin/swarm/capacity free KV tokens, GPUs, concurrency limits
  POST /api/admin/shutdown       graceful stop of a server started by serve()
  POST /api/admin/prune-history  drop stored responses by age and/or count
  GET  /api/admin/api-key        the key in force; POST /api-key/rotate issues a
                                 new one, in force from the next request
  POST /api/admin/ws-ticket      one-time 30 s ticket for /api/admin/ws?t=...

Every route needs the API key when one is configured (the guards treat
/api/admin like any other path).  Model download and Hugging Face search are
not offered: a node here fetches nothing.

Reference behaviour: src/api/admin.rs (stats, config get/update/reload,
models, diagnostics, performance, responses, storage breakdown, API key
rotation at :2318 -- there in force after a restart, here at once; routes at
src/api/server.rs:274-330); websocket tickets as src/api/middleware.rs:551.
"""
from __future__ import annotations

import os
import time

from fastapi import Request  # module level: route annotations resolve from globals


def register(app, S, settings, config_path: str | None = None):
    from .api import ApiError

    def engine():
        return S.ae.engine

    @app.get("/api/admin/stats")
    async def stats():
        out = S.ae.metrics.summary(60.0)
        e = engine()
        out.update(running=e.sched.num_running, waiting=e.sched.num_waiting,
                   kv_pages_free=e.bm.num_free(), kv_pages=e.bm.num_pages,
                   prefix_cache_hit_tokens=e.bm.prefix_hit_tokens, ready=S.ae.ready)
        return out

    @app.get("/api/admin/performance")
    async def performance():
        m = S.ae.metrics
        return {"windows": {str(int(w)): m.summary(w) for w in (10.0, 60.0, 300.0)}}

    def config_view() -> dict:
        e = engine()
        ec = {k: (list(v) if isinstance(v, tuple) else v) for k, v in vars(e.ecfg).items()}
        return {"engine": ec, "server": settings.public(), "model": e.cfg.name,
                "config_file": config_path}

    @app.get("/api/admin/config")
    async def get_config():
        return config_view()

    def apply(update: dict):
        bad = set(update) - {"rpm", "cors_origins", "max_body"}
        if bad:
            raise ApiError(400, f"not changeable at run time: {sorted(bad)} "
                                "(engine settings need a restart)")
        if "rpm" in update:
            v = int(update["rpm"])
            if v < 0:
                raise ApiError(400, "rpm must be >= 0")
            settings.rpm = v
        if "cors_origins" in update:
            o = update["cors_origins"]
            if not isinstance(o, list) or not all(isinstance(x, str) for x in o):
                raise ApiError(400, "cors_origins must be a list of strings")
            settings.cors_origins = tuple(o)
        if "max_body" in update:
            v = int(update["max_body"])
            if v < 1024:
                raise ApiError(400, "max_body must be at least 1024 bytes")
            settings.max_body = v

    @app.put("/api/admin/config")
    async def put_config(request: Request):
        body = await request.json()
        if not isinstance(body, dict):
            raise ApiError(400, "body must be an object")
        apply(body.get("server", body))
        return config_view()

    @app.post("/api/admin/config/reload")
    async def reload_config():
        if not config_path:
            raise ApiError(400, "the server was started without a config file")
        from ..utils.config import load_server_settings
        try:
            upd = load_server_settings(config_path)
        except (OSError, ValueError) as e:
            raise ApiError(400, f"cannot read {config_path}: {e}")
        apply(upd)
        return config_view()

    @app.get("/api/admin/models")
    async def models():
        e = engine()
        cfg = e.cfg
        m = e.model
        weight_bytes = 0
        types: dict = {}
        for lin in getattr(m, "_linears", lambda: [])():
            weight_bytes += lin.nbytes
            types[str(lin.qtype)] = types.get(str(lin.qtype), 0) + 1
        v = getattr(e, "vision", None)
        return {"model": cfg.name, "arch": cfg.arch, "layers": cfg.n_layers, "hidden": cfg.hidden,
                "vocab": cfg.vocab, "params": cfg.param_count(), "linear_weight_bytes": weight_bytes,
                "linear_types": types, "lora_adapters": [n for n in getattr(e, "lora_names", []) if n],
                "lora_slots": e.ecfg.max_loras,
                "vision": None if v is None else {"projector": v.cfg.projector,
                                                  "image_size": v.cfg.image_size,
                                                  "rows_per_image": v.rows_per_image},
                "ids": S.models()}

    @app.post("/api/admin/lora")
    async def load_lora(request: Request):
        body = await request.json()
        name, path = body.get("name"), body.get("path")
        if not name or not path:
            raise ApiError(400, "name and path are required")
        if not os.path.isfile(path):
            raise ApiError(404, f"no file {path}")
        try:
            n = await S.ae.call(lambda e: e.load_lora(path, name))
        except (RuntimeError, ValueError) as ex:
            raise ApiError(400, str(ex))
        return {"loaded": n, "models": S.models()}

    @app.get("/api/admin/adapters")
    async def adapters():
        e = engine()
        return {"data": [{"id": n, "slot": i, "model": f"{S.model_name}:{n}"}
                         for i, n in enumerate(getattr(e, "lora_names", [])) if n],
                "slots": e.ecfg.max_loras}

    @app.post("/api/admin/adapters")
    async def add_adapter(request: Request):
        return await load_lora(request)

    @app.delete("/api/admin/adapters/{name}")
    async def remove_adapter(name: str):
        try:
            slot = await S.ae.call(lambda e: e.unload_lora(name))
        except KeyError:
            raise ApiError(404, f"no adapter {name!r}")
        except RuntimeError as ex:
            raise ApiError(409, str(ex))
        return {"removed": name, "slot": slot, "models": S.models()}

    @app.get("/api/admin/models/{mid}")
    async def model_detail(mid: str):
        if mid not in S.models() and S.lora_of({"model": mid}) is None:
            raise ApiError(404, f"no model {mid!r}")
        d = await models()
        d["id"] = mid
        d["adapter"] = S.lora_of({"model": mid})
        return d

    @app.get("/api/admin/models/{mid}/status")
    async def model_status(mid: str):
        if mid not in S.models() and S.lora_of({"model": mid}) is None:
            raise ApiError(404, f"no model {mid!r}")
        return {"id": mid, "loaded": True, "ready": S.ae.ready}

    @app.get("/api/admin/version")
    async def version():
        import torch

        from .. import __version__
        return {"name": "swarmllm_b200", "version": __version__, "torch": torch.__version__,
                "cuda": torch.version.cuda}

    @app.get("/api/admin/peers")
    async def peers():
        # one node: the GPUs are ranks of this process group, not swarm peers
        return {"peers": [], "node": {"model": S.model_name, "ready": S.ae.ready}}

    @app.get("/api/admin/schedule")
    async def schedule():
        e = engine()
        ec = e.ecfg
        return {"running": e.sched.num_running, "waiting": e.sched.num_waiting,
                "preemptions": getattr(e.sched, "num_preemptions", 0), "steps": e.steps,
                "max_running": ec.max_running, "max_step_tokens": ec.max_step_tokens,
                "prefill_chunk": ec.prefill_chunk, "kv_pages_free": e.bm.num_free(),
                "kv_pages": e.bm.num_pages, "page_size": e.bm.page_size}

    @app.get("/api/admin/swarm/capacity")
    async def capacity():
        e = engine()
        import torch
        return {"gpus": torch.cuda.device_count() if torch.cuda.is_available() else 0,
                "kv_tokens_free": e.bm.num_free() * e.bm.page_size,
                "kv_tokens": e.bm.num_pages * e.bm.page_size,
                "running": e.sched.num_running, "max_running": e.ecfg.max_running,
                "max_model_len": e.ecfg.max_model_len}

    @app.post("/api/admin/shutdown")
    async def shutdown():
        hook = getattr(app.state, "shutdown_hook", None)
        if hook is None:
            raise ApiError(501, "this server was not started by serve(): no shutdown hook")
        hook()
        return {"status": "shutting down"}

    @app.get("/api/admin/diagnostics")
    async def diagnostics():
        from ..utils.diagnostics import collect
        return collect(engine())

    @app.get("/api/admin/responses")
    async def responses(limit: int = 50):
        store = getattr(app.state, "response_store", None)
        if store is None:
            return {"data": []}
        with store.lock:
            rows = store.db.execute("SELECT id, created FROM responses ORDER BY created DESC LIMIT ?",
                                    (max(1, min(1000, int(limit))),)).fetchall()
        return {"data": [{"id": r[0], "created": r[1]} for r in rows]}

    @app.post("/api/admin/prune-history")
    async def prune_history(request: Request):
        """Body {"older_than_days": d} and/or {"keep": n}: drop stored
        /v1/responses older than d days / all but the newest n."""
        body = await request.json() if await request.body() else {}
        store = getattr(app.state, "response_store", None)
        days, keep = body.get("older_than_days"), body.get("keep")
        if days is None and keep is None:
            raise ApiError(400, "give older_than_days and/or keep")
        for v in (days, keep):
            if v is not None and (not isinstance(v, (int, float)) or isinstance(v, bool) or v < 0):
                raise ApiError(400, "older_than_days and keep must be non-negative numbers")
        if store is None:
            return {"removed": 0, "left": 0}
        removed, left = store.prune(None if days is None else float(days) * 86400.0,
                                    None if keep is None else int(keep))
        return {"removed": removed, "left": left}

    # ------------------------------------------------------------------ API key
    @app.get("/api/admin/api-key")
    async def api_key():
        """The key in force (this route itself needs it when one is set)."""
        return {"auth_required": bool(settings.api_key), "api_key": settings.api_key or None,
                "key_file": settings.key_file}

    @app.post("/api/admin/api-key/rotate")
    async def rotate_api_key():
        """Issue a new random key; the old one stops working with the next
        request (no restart), and outstanding websocket tickets are dropped."""
        key = settings.rotate_key()
        return {"api_key": key, "effective": "now", "key_file": settings.key_file}

    @app.post("/api/admin/ws-ticket")
    async def ws_ticket():
        """A one-time, 30-second ticket for /api/admin/ws?t=<ticket>."""
        return {"ticket": settings.issue_ticket(), "expires_in_s": settings.TICKET_S}

    @app.get("/api/admin/storage/breakdown")
    @app.get("/api/admin/storage")
    async def storage():
        src = getattr(engine(), "source_path", None)
        files = []
        if src:
            paths = [os.path.join(src, f) for f in sorted(os.listdir(src))] if os.path.isdir(src) else [src]
            for f in paths:
                if os.path.isfile(f):
                    files.append({"path": f, "bytes": os.path.getsize(f)})
        return {"source": src, "files": files, "total_bytes": sum(f["bytes"] for f in files)}
