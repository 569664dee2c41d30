"""Request traces, the stage profiler, NVTX ranges and device timers.

* ``RequestTrace``   one record per request: arrival, first token (TTFT),
                     per-token gaps (TPOT); the single source for logs, the
                     Prometheus histograms and HTTP response headers
                     (reference: src/inference/trace.rs:1-70).
* ``StageProfiler``  ``SWARMLLM_PROFILE=1`` turns on per-stage wall-clock
                     accounting; ``SWARMLLM_PROFILE_SYNC=1`` synchronises the
                     device around each stage so the numbers are device time
                     (reference: src/inference/prof.rs:1-60).  Stages are also
                     NVTX ranges, visible in any CUDA timeline tool.
* ``device_timer``   CUDA-event timing on the launching stream.
"""
from __future__ import annotations

import contextlib
import os
import time
from dataclasses import dataclass, field

import torch


@dataclass
class RequestTrace:
    request_id: int
    prompt_len: int
    route: str = "local"
    t_arrival: float = field(default_factory=time.perf_counter)
    t_first: float | None = None
    t_last: float | None = None
    t_done: float | None = None
    n_tokens: int = 0
    gaps: list = field(default_factory=list)

    def on_token(self, now: float):
        if self.t_first is None:
            self.t_first = now
        elif self.t_last is not None:
            self.gaps.append(now - self.t_last)
        self.t_last = now
        self.n_tokens += 1

    def finish(self, now: float):
        self.t_done = now

    @property
    def ttft(self) -> float | None:
        return None if self.t_first is None else self.t_first - self.t_arrival

    @property
    def tpot(self) -> float | None:
        return sum(self.gaps) / len(self.gaps) if self.gaps else None

    def headers(self) -> dict:
        h = {"x-swarmllm-route": self.route, "x-swarmllm-tokens": str(self.n_tokens)}
        if self.ttft is not None:
            h["x-swarmllm-ttft-ms"] = f"{self.ttft * 1e3:.2f}"
        if self.tpot is not None:
            h["x-swarmllm-tpot-ms"] = f"{self.tpot * 1e3:.2f}"
        return h


class StageProfiler:
    def __init__(self, enabled: bool | None = None, sync: bool | None = None):
        self.enabled = (os.environ.get("SWARMLLM_PROFILE") == "1") if enabled is None else enabled
        self.sync = (os.environ.get("SWARMLLM_PROFILE_SYNC") == "1") if sync is None else sync
        self.totals: dict[str, float] = {}
        self.counts: dict[str, int] = {}

    @contextlib.contextmanager
    def stage(self, name: str):
        if not self.enabled:
            yield
            return
        cuda = torch.cuda.is_available()
        if cuda:
            torch.cuda.nvtx.range_push(name)
            if self.sync:
                torch.cuda.synchronize()
        t0 = time.perf_counter()
        try:
            yield
        finally:
            if cuda and self.sync:
                torch.cuda.synchronize()
            dt = time.perf_counter() - t0
            if cuda:
                torch.cuda.nvtx.range_pop()
            self.totals[name] = self.totals.get(name, 0.0) + dt
            self.counts[name] = self.counts.get(name, 0) + 1

    def report(self) -> str:
        lines = [f"{k:24s} {v * 1e3:10.3f} ms  x{self.counts[k]}" for k, v in
                 sorted(self.totals.items(), key=lambda kv: -kv[1])]
        return "\n".join(lines)


@contextlib.contextmanager
def device_timer(out: list, stream: torch.cuda.Stream | None = None):
    """Append the elapsed device milliseconds of the enclosed work to `out`."""
    s = stream or torch.cuda.current_stream()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a.record(s)
    yield
    b.record(s)
    torch.cuda.synchronize()
    out.append(a.elapsed_time(b))
