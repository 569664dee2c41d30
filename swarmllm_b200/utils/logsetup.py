"""Logging: the "swarmllm_b200" logger to stderr and, optionally, a rotating
file (50 MB x 3 by default), as text or one JSON object per line.

Reference behaviour: src/logging.rs:57,150 (tracing subscriber, rotating file,
JSON or pretty format).
"""
from __future__ import annotations

import json
import logging
import logging.handlers
import time

LOGGER = "swarmllm_b200"


class JsonFormatter(logging.Formatter):
    def format(self, rec: logging.LogRecord) -> str:
        d = {"ts": round(rec.created, 3), "time": time.strftime("%Y-%m-%dT%H:%M:%S", time.gmtime(rec.created)),
             "level": rec.levelname.lower(), "logger": rec.name, "msg": rec.getMessage()}
        for k, v in getattr(rec, "fields", {}).items():
            d[k] = v
        if rec.exc_info:
            d["exc"] = self.formatException(rec.exc_info)
        return json.dumps(d)


_LEVELS = {"trace": logging.DEBUG, "debug": logging.DEBUG, "info": logging.INFO,
           "warn": logging.WARNING, "warning": logging.WARNING, "error": logging.ERROR}


def setup_logging(verbosity: int = 0, log_file: str | None = None, json_format: bool = False,
                  max_bytes: int = 50 << 20, backups: int = 3,
                  level: str | None = None) -> logging.Logger:
    """verbosity 0: info (or `level`), 1+: debug.  Idempotent: replaces this
    logger's handlers."""
    log = logging.getLogger(LOGGER)
    log.setLevel(logging.DEBUG if verbosity > 0 else _LEVELS.get(level or "info", logging.INFO))
    for h in list(log.handlers):
        log.removeHandler(h)
        h.close()
    fmt = JsonFormatter() if json_format else logging.Formatter(
        "%(asctime)s %(levelname).1s %(name)s: %(message)s")
    sh = logging.StreamHandler()
    sh.setFormatter(fmt)
    log.addHandler(sh)
    if log_file:
        fh = logging.handlers.RotatingFileHandler(log_file, maxBytes=max_bytes, backupCount=backups)
        fh.setFormatter(fmt)
        log.addHandler(fh)
    log.propagate = False
    return log


def get_logger(sub: str | None = None) -> logging.Logger:
    return logging.getLogger(LOGGER if not sub else f"{LOGGER}.{sub}")
