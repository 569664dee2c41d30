"""Request-level data parallelism: R engine replicas, one front scheduler.

Each replica is a process that owns a whole engine (one GPU, or the host CPU)
and runs its own continuous-batching loop; the front keeps the request table
and decides, per request, which replica serves it:

* prefix affinity first -- a request whose first `affinity_tokens` tokens
  match a recent request's goes to the same replica, whose prefix cache holds
  those pages, unless that replica is more than `slack` tokens of work ahead
  of the least loaded one;
* else the least loaded replica, by outstanding work (prompt tokens not yet
  answered plus tokens still to generate).

`ReplicaSet` offers the engine interface the HTTP server drives
(`add_request`, `step`, `abort`, `release`, `has_work`, `traces`, and `sched` /
`bm` views summed over the replicas), so `serve --replicas N` puts it where a
single engine would be.  The reference gets the same effect from many peers
each serving whole requests, its router picking one per request and pricing
cached prefixes (src/inference/router/mod.rs:1270,
src/inference/scheduler/cached_prefix.rs:253).
"""
from __future__ import annotations

import collections
import itertools
import queue
import time
from dataclasses import dataclass, field

from ..utils.tracing import RequestTrace


def engine_factory(spec: dict, idx: int):
    """Build replica `idx`'s engine from a picklable spec: {"preset" or
    "gguf", "device": "cuda" | "cpu", "ecfg": EngineConfig, "seed"}; CUDA
    replicas take GPU `idx`."""
    from ..engine import LLMEngine
    from ..models.config import preset
    dev = f"cuda:{idx}" if spec.get("device", "cpu") == "cuda" else "cpu"
    if dev.startswith("cuda"):
        import torch
        torch.cuda.set_device(idx)
    if spec.get("gguf"):
        return LLMEngine.from_gguf(spec["gguf"], dev, spec.get("ecfg"))
    cfg = spec["cfg"] if spec.get("cfg") is not None else preset(spec["preset"])
    return LLMEngine.from_config(cfg, dev, spec.get("ecfg"), seed=spec.get("seed", 0))


def _stats(eng) -> dict:
    return {"running": eng.sched.num_running, "waiting": eng.sched.num_waiting,
            "free_pages": eng.bm.num_free(), "pages": eng.bm.num_pages,
            "hits": eng.bm.prefix_hit_tokens,
            "preemptions": getattr(eng.sched, "num_preemptions", 0), "steps": eng.steps}


def _replica_main(idx: int, factory, spec, inbox, outbox):
    """A replica's loop: commands from the front between steps, outputs back."""
    try:
        eng = factory(spec, idx)
    except Exception as e:  # noqa: BLE001 -- reported to the front
        outbox.put(("dead", idx, f"engine construction failed: {e!r}", []))
        return
    outbox.put(("ready", idx, _stats(eng)))
    live: set = set()
    while True:
        block = not eng.has_work()
        try:
            cmd = inbox.get(timeout=0.05) if block else inbox.get_nowait()
        except queue.Empty:
            cmd = None
        while cmd is not None:
            op = cmd[0]
            if op == "stop":
                return
            try:
                if op == "add":
                    _, prompt, params, rid, kw = cmd
                    eng.add_request(prompt, params, request_id=rid, **kw)
                    live.add(rid)
                elif op == "abort":
                    eng.abort(cmd[1])
                    live.discard(cmd[1])
                elif op == "release":
                    eng.release(cmd[1])
            except Exception as e:  # noqa: BLE001 -- a bad request fails alone
                if op == "add":
                    outbox.put(("reject", idx, cmd[3], repr(e)))
            try:
                cmd = inbox.get_nowait()
            except queue.Empty:
                cmd = None
        if not eng.has_work():
            continue
        try:
            outs = eng.step()
        except Exception as e:  # noqa: BLE001 -- the front fails this replica's requests
            outbox.put(("dead", idx, repr(e), sorted(live)))
            return
        for rid, _tok, fin in outs:
            if fin:
                live.discard(rid)
        outbox.put(("out", idx, outs, _stats(eng)))


class _Sum:
    """Scheduler / block-manager numbers summed over the replicas (the
    attributes the status routes and /metrics read)."""

    def __init__(self, rs: "ReplicaSet"):
        self._rs = rs

    def _sum(self, k):
        return sum(s.get(k, 0) for s in self._rs.stats)

    num_running = property(lambda self: self._sum("running"))
    num_waiting = property(lambda self: self._sum("waiting"))
    num_preemptions = property(lambda self: self._sum("preemptions"))
    num_pages = property(lambda self: self._sum("pages"))
    prefix_hit_tokens = property(lambda self: self._sum("hits"))

    def num_free(self):
        return self._sum("free_pages")


@dataclass
class _Req:
    replica: int
    work: int                      # prompt tokens + tokens still to generate
    tokens: list = field(default_factory=list)
    finished: bool = False
    error: str | None = None


@dataclass
class ReplicaOutput:
    request_id: int
    prompt_len: int
    token_ids: list
    finished: bool
    replica: int


class ReplicaSet:
    def __init__(self, cfg, spec: dict, n: int, factory=engine_factory, ecfg=None,
                 affinity_tokens: int = 64, slack: int = 4096, start_method: str = "spawn",
                 ready_timeout_s: float = 600.0):
        import multiprocessing as mp
        self.cfg, self.ecfg, self.n = cfg, ecfg if ecfg is not None else spec.get("ecfg"), n
        self.affinity_tokens, self.slack = affinity_tokens, slack
        ctx = mp.get_context(start_method)
        self._out = ctx.Queue()
        self._in = [ctx.Queue() for _ in range(n)]
        self._procs = [ctx.Process(target=_replica_main, args=(i, factory, spec, self._in[i],
                                                                self._out), daemon=True)
                       for i in range(n)]
        for p in self._procs:
            p.start()
        self.stats = [dict() for _ in range(n)]
        self.dead: dict[int, str] = {}
        self.reqs: dict[int, _Req] = {}
        self.traces: dict[int, RequestTrace] = {}
        self._affinity: collections.OrderedDict = collections.OrderedDict()
        self._ids = itertools.count()
        self._pending: list = []
        self.sched = self.bm = _Sum(self)
        deadline = time.monotonic() + ready_timeout_s
        ready = set()
        while len(ready) + len(self.dead) < n:
            left = deadline - time.monotonic()
            if left <= 0:
                raise TimeoutError(f"replicas not ready: {sorted(set(range(n)) - ready)}")
            try:
                msg = self._out.get(timeout=min(left, 1.0))
            except queue.Empty:
                for i, p in enumerate(self._procs):
                    if not p.is_alive() and i not in ready and i not in self.dead:
                        self.dead[i] = f"exited with {p.exitcode} before it was ready"
                continue
            if msg[0] == "ready":
                ready.add(msg[1])
                self.stats[msg[1]] = msg[2]
            elif msg[0] == "dead":
                self.dead[msg[1]] = msg[2]
            else:
                self._pending.append(msg)
        if not ready:
            raise RuntimeError(f"no replica came up: {self.dead}")

    # ------------------------------------------------------------------ engine interface
    @property
    def steps(self) -> int:
        return sum(s.get("steps", 0) for s in self.stats)

    def load(self, i: int) -> int:
        return sum(r.work for r in self.reqs.values() if r.replica == i and not r.finished)

    def _choose(self, prompt) -> int:
        alive = [i for i in range(self.n) if i not in self.dead]
        if not alive:
            raise RuntimeError(f"every replica failed: {self.dead}")
        loads = {i: self.load(i) for i in alive}
        least = min(alive, key=lambda i: (loads[i], i))
        if len(prompt) >= self.affinity_tokens:
            key = hash(tuple(prompt[: self.affinity_tokens]))
            i = self._affinity.get(key)
            if i is not None and i in loads and loads[i] <= loads[least] + self.slack:
                self._affinity.move_to_end(key)
                return i
            self._affinity[key] = least
            if len(self._affinity) > 4096:
                self._affinity.popitem(last=False)
        return least

    def add_request(self, prompt_ids, params=None, request_id: int | None = None, **kw) -> int:
        from ..engine.sampling import SamplingParams
        params = params or SamplingParams()
        rid = next(self._ids) if request_id is None else int(request_id)
        prompt = [int(t) for t in prompt_ids]
        i = self._choose(prompt)
        self.reqs[rid] = _Req(i, len(prompt) + int(params.max_tokens))
        self.traces[rid] = RequestTrace(rid, len(prompt), route=f"replica{i}")
        self._in[i].put(("add", prompt, params, rid, kw))
        return rid

    def abort(self, rid: int):
        r = self.reqs.get(rid)
        if r is not None and not r.finished:
            r.finished = True
            self._in[r.replica].put(("abort", rid))

    def release(self, rid: int):
        r = self.reqs.pop(rid, None)
        self.traces.pop(rid, None)
        if r is not None and r.replica not in self.dead:
            self._in[r.replica].put(("release", rid))

    def has_work(self) -> bool:
        return any(not r.finished for r in self.reqs.values())

    def error_of(self, rid: int) -> str | None:
        r = self.reqs.get(rid)
        return None if r is None else r.error

    def output(self, rid: int) -> list:
        return list(self.reqs[rid].tokens)

    def step(self, wait_s: float = 0.02) -> list:
        """Outputs (rid, token, finished) that arrived from any replica since
        the last call; waits up to `wait_s` for the first when none is queued."""
        msgs, self._pending = self._pending, []
        try:
            if not msgs:
                msgs.append(self._out.get(timeout=wait_s))
            while True:
                msgs.append(self._out.get_nowait())
        except queue.Empty:
            pass
        outs, now = [], time.perf_counter()
        for m in msgs:
            kind, i = m[0], m[1]
            if kind == "out":
                self.stats[i] = m[3]
                for rid, tok, fin in m[2]:
                    r = self.reqs.get(rid)
                    if r is None or r.finished:
                        continue
                    r.tokens.append(tok)
                    r.work = max(0, r.work - 1)
                    tr = self.traces.get(rid)
                    if tr is not None:
                        tr.on_token(now)
                    if fin:
                        r.finished = True
                    outs.append((rid, tok, fin))
            elif kind == "reject":
                r = self.reqs.get(m[2])
                if r is not None:
                    r.finished, r.error = True, m[3]
                    outs.append((m[2], None, True))
            elif kind == "dead":
                self.dead[i] = m[2]
                for rid, r in self.reqs.items():
                    if r.replica == i and not r.finished:
                        r.finished, r.error = True, f"replica {i} failed: {m[2]}"
                        outs.append((rid, None, True))
        # a replica that died without a word
        for i, p in enumerate(self._procs):
            if i not in self.dead and not p.is_alive():
                self.dead[i] = f"exited with {p.exitcode}"
                for rid, r in self.reqs.items():
                    if r.replica == i and not r.finished:
                        r.finished, r.error = True, f"replica {i} {self.dead[i]}"
                        outs.append((rid, None, True))
        return [o for o in outs if o[1] is not None or o[2]]

    def generate(self, prompts, params=None) -> list[ReplicaOutput]:
        rids = [self.add_request(p, params) for p in prompts]
        pending = set(rids)
        while pending:
            for rid, _tok, fin in self.step(0.1):
                if fin:
                    pending.discard(rid)
        out = []
        for rid, p in zip(rids, prompts):
            r = self.reqs[rid]
            if r.error:
                raise RuntimeError(r.error)
            out.append(ReplicaOutput(rid, len(p), list(r.tokens), True, r.replica))
            self.release(rid)
        return out

    def close(self, timeout_s: float = 30.0):
        for i in range(self.n):
            if i not in self.dead:
                try:
                    self._in[i].put(("stop",))
                except Exception:  # noqa: BLE001
                    pass
        for p in self._procs:
            p.join(timeout=timeout_s)
            if p.is_alive():
                p.terminate()
                p.join(timeout=5)
