"""Prometheus metrics (reference names: src/api/metrics.rs:303-924,
e.g. swarmllm_inference_requests_total, swarmllm_inference_latency_seconds).
Each server owns a private registry, so several engines in one process (tests)
do not collide."""
from __future__ import annotations

import collections
import time

from prometheus_client import CollectorRegistry, Counter, Gauge, Histogram, generate_latest


class Metrics:
    def __init__(self):
        r = self.registry = CollectorRegistry()
        self.req_total = Counter("swarmllm_inference_requests_total", "Requests started", registry=r)
        self.req_done = Counter("swarmllm_inference_requests_completed_total", "Requests completed",
                                registry=r)
        self.tokens = Counter("swarmllm_tokens_generated_total", "Tokens generated", registry=r)
        self.latency = Histogram("swarmllm_inference_latency_seconds", "Request latency", registry=r,
                                 buckets=(0.05, 0.1, 0.25, 0.5, 1, 2, 5, 10, 30, 60, 120))
        self.ttft = Histogram("swarmllm_time_to_first_token_seconds", "Time to first token", registry=r,
                              buckets=(0.01, 0.025, 0.05, 0.1, 0.25, 0.5, 1, 2, 5, 10))
        self.tpot = Histogram("swarmllm_time_per_output_token_seconds", "Mean gap between tokens",
                              registry=r, buckets=(0.002, 0.005, 0.01, 0.02, 0.05, 0.1, 0.25, 0.5))
        self.step_s = Histogram("swarmllm_engine_step_seconds", "Engine step time", registry=r,
                                buckets=(0.001, 0.0025, 0.005, 0.01, 0.025, 0.05, 0.1, 0.25, 0.5, 1))
        self.kv_free = Gauge("swarmllm_kv_pages_free", "Free KV pages", registry=r)
        self.kv_total = Gauge("swarmllm_kv_pages_total", "KV pages", registry=r)
        self.running = Gauge("swarmllm_requests_running", "Requests in the running batch", registry=r)
        self.waiting = Gauge("swarmllm_requests_waiting", "Requests waiting for admission",
                             registry=r)
        self.prefix_hits = Gauge("swarmllm_prefix_cache_hit_tokens",
                                 "Prompt tokens served from the prefix cache since start", registry=r)
        self.preemptions = Gauge("swarmllm_preemptions", "Requests preempted since start", registry=r)
        self.ready = Gauge("swarmllm_ready", "1 when the node accepts inference", registry=r)
        self.segments = Gauge("swarmllm_segments_served_total",
                              "Layer-range forwards run by this rank's pipeline stage", registry=r)
        self.net_bytes = Gauge("swarmllm_network_bytes_total",
                               "Bytes this rank sent to other ranks", registry=r)
        # recent window for the admin views: (wall time, step seconds, tokens), TTFTs
        self.recent_steps: collections.deque = collections.deque(maxlen=4096)
        self.recent_ttft: collections.deque = collections.deque(maxlen=1024)
        self.n_started = self.n_done = self.n_tokens = 0
        self.t0 = time.time()

    def set_engine(self, engine, ready: bool):
        """Scheduler and cache state, read when /metrics is scraped."""
        self.running.set(engine.sched.num_running)
        self.waiting.set(engine.sched.num_waiting)
        self.prefix_hits.set(engine.bm.prefix_hit_tokens)
        self.preemptions.set(getattr(engine.sched, "num_preemptions", 0))
        self.ready.set(1 if ready else 0)
        self.segments.set(getattr(engine, "segments_served", engine.steps))
        self.net_bytes.set(getattr(engine, "bytes_sent", 0))

    def requests_started(self):
        self.req_total.inc()
        self.n_started += 1

    def step(self, seconds: float, n_tokens: int):
        self.step_s.observe(seconds)
        self.recent_steps.append((time.time(), seconds, n_tokens))
        if n_tokens:
            self.tokens.inc(n_tokens)
            self.n_tokens += n_tokens

    def summary(self, window_s: float = 60.0) -> dict:
        """Totals, and rates over the last `window_s` seconds."""
        now = time.time()
        rec = [x for x in self.recent_steps if now - x[0] <= window_s]
        busy = sum(x[1] for x in rec)
        toks = sum(x[2] for x in rec)
        tt = sorted(self.recent_ttft)
        pct = lambda q: round(tt[min(len(tt) - 1, int(q * len(tt)))] * 1e3, 2) if tt else None
        return {"uptime_s": round(now - self.t0, 1), "requests_started": self.n_started,
                "requests_completed": self.n_done, "tokens_generated": self.n_tokens,
                "window_s": window_s, "window_steps": len(rec), "window_tokens": toks,
                "window_tok_s": round(toks / window_s, 2),
                "busy_fraction": round(min(1.0, busy / window_s), 4),
                "step_ms_mean": round(busy / len(rec) * 1e3, 3) if rec else None,
                "ttft_ms_p50": pct(0.5), "ttft_ms_p99": pct(0.99)}

    def request_done(self, tr):
        self.req_done.inc()
        self.n_done += 1
        if tr.ttft is not None:
            self.recent_ttft.append(tr.ttft)
        if tr.t_done is not None:
            self.latency.observe(tr.t_done - tr.t_arrival)
        if tr.ttft is not None:
            self.ttft.observe(tr.ttft)
        if tr.tpot is not None:
            self.tpot.observe(tr.tpot)

    def set_kv(self, free: int, total: int):
        self.kv_free.set(free)
        self.kv_total.set(total)

    def render(self) -> str:
        return generate_latest(self.registry).decode()
