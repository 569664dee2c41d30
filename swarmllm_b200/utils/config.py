"""Engine configuration from a TOML file and SWARMLLM_* environment variables.

The reference keeps its inference flags in a TOML [inference] section
(config/default.toml:10-172; src/config/inference.rs:19-686) with env
overrides.  Names kept where the meaning matches:

  [inference]
  continuous_batching = true      (always on here)
  prefill_chunk_tokens = 2048     -> EngineConfig.prefill_chunk
  max_concurrent_decode_batch     -> EngineConfig.max_running
  max_seq_len_override            -> EngineConfig.max_model_len
  prefix_cache_enabled            -> EngineConfig.prefix_cache
  cuda_graphs (SWARMLLM_CUDA_GRAPH=0 disables)
  draft_model_path                -> EngineConfig.draft_model (speculative serving; also a
                                     preset name, "self" or "ngram")
  speculative_gamma = 4           -> EngineConfig.spec_depth (draft tree depth)
  speculative_width = 4           -> EngineConfig.spec_width (children kept per level)
  cpu_native = false              -> EngineConfig.cpu_native (CPU device: quantized weights
                                     through the native int8 matmul and paged attention)

Environment: SWARMLLM_MAX_MODEL_LEN, SWARMLLM_MAX_RUNNING, SWARMLLM_PREFILL_CHUNK,
SWARMLLM_KV_PAGES, SWARMLLM_KV_FRACTION, SWARMLLM_PREFIX_CACHE, SWARMLLM_CUDA_GRAPH,
SWARMLLM_CPU_NATIVE.

A [server] table (rpm, cors_origins, max_body) holds the request-guard
settings; the admin API re-reads it on /api/admin/config/reload.

A [logging] table (the reference's names: level = trace|debug|info|warn|error,
format = pretty|json; plus file = a rotating log file) sets up logging when
the command line does not.
"""
from __future__ import annotations

import os

from ..engine.engine import EngineConfig

_TOML_KEYS = {
    "prefill_chunk_tokens": "prefill_chunk",
    "max_concurrent_decode_batch": "max_running",
    "max_seq_len_override": "max_model_len",
    "prefix_cache_enabled": "prefix_cache",
    "max_step_tokens": "max_step_tokens",
    "kv_pages": "kv_pages",
    "kv_fraction": "kv_fraction",
    "cuda_graphs": "cuda_graphs",
    "page_size": "page_size",
    "draft_model_path": "draft_model",      # drafter GGUF (or preset / "self" / "ngram")
    "speculative_gamma": "spec_depth",      # draft depth (tokens guessed per round)
    "speculative_width": "spec_width",
    "cpu_native": "cpu_native",
}

_ENV = {
    "SWARMLLM_MAX_MODEL_LEN": ("max_model_len", int),
    "SWARMLLM_MAX_RUNNING": ("max_running", int),
    "SWARMLLM_PREFILL_CHUNK": ("prefill_chunk", int),
    "SWARMLLM_MAX_STEP_TOKENS": ("max_step_tokens", int),
    "SWARMLLM_KV_PAGES": ("kv_pages", int),
    "SWARMLLM_KV_FRACTION": ("kv_fraction", float),
    "SWARMLLM_PREFIX_CACHE": ("prefix_cache", lambda v: v not in ("0", "false", "False")),
    "SWARMLLM_CUDA_GRAPH": ("cuda_graphs", lambda v: v not in ("0", "false", "False")),
    "SWARMLLM_DRAFT_MODEL": ("draft_model", str),
    "SWARMLLM_SPEC_DEPTH": ("spec_depth", int),
    "SWARMLLM_SPEC_WIDTH": ("spec_width", int),
    "SWARMLLM_CPU_NATIVE": ("cpu_native", lambda v: v not in ("0", "false", "False")),
}


def load_engine_config(path: str | None = None, env=None) -> EngineConfig:
    cfg = EngineConfig()
    if path:
        import tomllib
        with open(path, "rb") as f:
            data = tomllib.load(f)
        inf = data.get("inference", data)
        for k, v in inf.items():
            attr = _TOML_KEYS.get(k)
            if attr is not None:
                setattr(cfg, attr, type(getattr(cfg, attr))(v))
    env = os.environ if env is None else env
    for k, (attr, conv) in _ENV.items():
        if k in env:
            setattr(cfg, attr, conv(env[k]))
    if cfg.max_step_tokens < cfg.prefill_chunk:
        cfg.max_step_tokens = cfg.prefill_chunk
    return cfg


def load_logging_settings(path: str | None) -> dict:
    """level / format / file from a TOML [logging] table ({} without one)."""
    if not path:
        return {}
    import tomllib
    with open(path, "rb") as f:
        lg = tomllib.load(f).get("logging", {})
    out = {}
    if lg.get("level") in ("trace", "debug", "info", "warn", "warning", "error"):
        out["level"] = lg["level"]
    if lg.get("format") in ("pretty", "json"):
        out["json"] = lg["format"] == "json"
    if isinstance(lg.get("file"), str) and lg["file"]:
        out["file"] = lg["file"]
    return out


def load_server_settings(path: str) -> dict:
    """Guard settings from a TOML [server] table (rpm, cors_origins, max_body),
    the ones the admin API can apply at run time."""
    import tomllib
    with open(path, "rb") as f:
        doc = tomllib.load(f)
    srv = doc.get("server", {})
    return {k: srv[k] for k in ("rpm", "cors_origins", "max_body") if k in srv}
