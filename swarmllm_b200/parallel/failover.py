"""Failure detection and recovery for the pipeline-parallel engine.

A control TCPStore (hosted by the root rank, separate from the process
groups) outlives every process group.  Ranks heartbeat into it once per
engine step.  When a collective fails -- a peer's process died (gloo reports
the closed connection at once) or stopped answering (the group's short
timeout) -- or the root sees a stale heartbeat:

  1. every survivor drops the broken process group and registers itself
     under the next membership epoch;
  2. the root waits a grace period, fixes the membership (the ranks that
     registered) and publishes it;
  3. the survivors form a new process group through a store prefix for that
     epoch and rebuild the pipeline over the survivors: new stage boundaries
     from the layer planner, each rank reloading its new layer range;
  4. the root replays every unfinished request as (prompt + tokens generated
     so far) with the remaining token budget: the lost KV is recomputed, so
     greedy output is identical to an undisturbed run.

The root holds the scheduler; if the root itself fails the requests are lost
(the client retries), as when the reference's coordinator fails.

Reference behaviour: HealthMonitor pings and missed-ping death
(src/health/monitor.rs:702-704,904), router retry with re-planning
(src/inference/router/mod.rs:524,598,659), failover_segment onto standbys and
replay of retained activations (src/inference/pipeline/distributed.rs:2461).

Ranks that fail repeatedly (missing at a recovery, or stale while alive) are
ejected for a while by an OutlierTracker and left out of the membership.
"""
from __future__ import annotations

import datetime
import time
from dataclasses import dataclass, field

import torch.distributed as dist

from ..engine.sampling import SamplingParams


@dataclass
class _Req:
    prompt: list
    params: SamplingParams
    out: list = field(default_factory=list)
    done: bool = False


class RankFailure(RuntimeError):
    pass


class OutlierTracker:
    """Failure counts per rank over a sliding window.  A rank with `limit`
    failures inside `window_s` is ejected for `eject_s`: the root leaves it
    out of the next memberships even if it registers as alive (a straggler
    whose heartbeat keeps going stale, a rank that keeps breaking the group).
    Reference behaviour: peers that keep failing a model are left out for a
    while (src/daemon/state/peer_outliers.rs:60-106)."""

    def __init__(self, limit: int = 2, window_s: float = 600.0, eject_s: float = 1800.0,
                 clock=time.monotonic):
        self.limit, self.window_s, self.eject_s, self.clock = limit, window_s, eject_s, clock
        self._fails: dict[int, list[float]] = {}
        self._until: dict[int, float] = {}

    def record(self, rank: int):
        now = self.clock()
        f = [t for t in self._fails.get(rank, []) if now - t <= self.window_s] + [now]
        self._fails[rank] = f
        if len(f) >= self.limit:
            self._until[rank] = now + self.eject_s
            self._fails[rank] = []

    def ejected(self) -> set[int]:
        now = self.clock()
        for r in [r for r, t in self._until.items() if t <= now]:
            del self._until[r]
        return set(self._until)

    def members(self, alive: list[int]) -> list[int]:
        """The next membership: alive ranks minus the ejected ones (never
        empty: the ranks asking are alive, so the first of them stays)."""
        out = [r for r in alive if r not in self.ejected()]
        return out or alive[:1]


class ResilientPipeline:
    def __init__(self, build_engine, rank: int, world: int, ctl_host: str, ctl_port: int,
                 backend: str = "gloo", pg_timeout_s: float = 10.0, grace_s: float | None = None,
                 heartbeat_stale_s: float = 30.0, outliers: OutlierTracker | None = None):
        """`build_engine()` returns a pipeline engine over the current default
        process group -- the synchronous PipelineEngine (collective step()) or
        the wave-pipelined AsyncPipelineEngine (collective run()); it is called
        again after every re-plan."""
        self.rank, self.world0 = rank, world
        self.backend, self.pg_timeout_s = backend, pg_timeout_s
        # a survivor that only learns of the failure from the group timeout
        # must still register before the root fixes the membership
        self.grace_s = grace_s if grace_s is not None else pg_timeout_s + 2.0
        self.stale_s = heartbeat_stale_s
        self.store = dist.TCPStore(ctl_host, ctl_port, world, rank == 0,
                                   timeout=datetime.timedelta(seconds=60))
        self.members = list(range(world))
        self.epoch = 0
        self.build_engine = build_engine
        self.recoveries = 0
        self.rebalances = 0
        self.outliers = outliers or OutlierTracker()
        self._suspects: list[int] = []     # stale ranks seen by the root before a recovery
        self._form_group()
        self.eng = build_engine()

    # ------------------------------------------------------------------ membership
    @property
    def root(self) -> bool:
        return self.rank == self.members[0]

    def _form_group(self):
        pre = dist.PrefixStore(f"pg{self.epoch}", self.store)
        dist.init_process_group(self.backend, store=pre, rank=self.members.index(self.rank),
                                world_size=len(self.members),
                                timeout=datetime.timedelta(seconds=self.pg_timeout_s))

    def _heartbeat(self, step: int):
        self.store.set(f"hb/{self.rank}", f"{step}:{time.time()}")

    def stale_ranks(self) -> list[int]:
        """Members whose last heartbeat is older than the staleness limit."""
        now, bad = time.time(), []
        for r in self.members:
            if r == self.rank:
                continue
            try:
                ts = float(self.store.get(f"hb/{r}").decode().split(":")[1])
            except Exception:
                continue
            if now - ts > self.stale_s:
                bad.append(r)
        return bad

    def _recover(self):
        self.recoveries += 1
        try:
            dist.destroy_process_group()
        except Exception:
            pass
        self.epoch += 1
        self.store.set(f"alive/{self.epoch}/{self.rank}", "1")
        key = f"members/{self.epoch}"
        if self.rank == self.members[0]:
            time.sleep(self.grace_s)
            alive = [r for r in self.members
                     if self.store.check([f"alive/{self.epoch}/{r}"])]
            for r in self.members:
                if r not in alive or r in self._suspects:
                    self.outliers.record(r)
            self._suspects = []
            self.store.set(key, ",".join(map(str, self.outliers.members(alive))))
        self.store.wait([key], datetime.timedelta(seconds=60))
        self.members = [int(x) for x in self.store.get(key).decode().split(",")]
        if self.rank not in self.members:
            raise RankFailure("this rank was dropped from the membership")
        self._form_group()
        self.eng = self.build_engine()

    # ------------------------------------------------------------------ generation
    def generate(self, prompts: list[list[int]], params: SamplingParams | None = None,
                 max_recoveries: int = 3):
        """Collective over the survivors; the root returns the token lists."""
        params = params or SamplingParams()
        reqs = [_Req(list(p), params) for p in prompts] if self.root else []
        step = 0
        while True:
            try:
                rid_of = {}
                if self.root:
                    for i, r in enumerate(reqs):
                        left = r.params.max_tokens - len(r.out)
                        if r.done or left <= 0:
                            r.done = True
                            continue
                        sp = SamplingParams(**{**r.params.__dict__, "max_tokens": left})
                        rid_of[self.eng.add_request(r.prompt + r.out, sp)] = i
                def take(events):
                    for rid, tok, fin in events:
                        r = reqs[rid_of[rid]]
                        r.out.append(tok)
                        r.done = r.done or fin

                def beat():
                    nonlocal step
                    step += 1
                    self._heartbeat(step)
                    if self.root:
                        stale = self.stale_ranks()
                        if stale:
                            self._suspects = stale
                            raise RankFailure(f"stale heartbeat: {stale}")
                if hasattr(self.eng, "run"):   # wave-pipelined engine: one collective run
                    self.eng.run(on_events=take if self.root else None, on_step=beat)
                else:
                    while self.eng.has_work():
                        take(self.eng.step())
                        beat()
                return [r.out for r in reqs] if self.root else None
            except (RuntimeError, dist.DistBackendError):
                if self.recoveries >= max_recoveries:
                    raise
                self._recover()

    def rebalance(self, rebalancer, stage_s: list | None = None) -> bool:
        """Collective: gather every stage's measured step time (or use
        `stage_s`), let the root ask `rebalancer` (parallel/rebalance.py) for
        a better cut, and rebuild every rank's engine with it.  `build_engine`
        must accept `bounds=`.  Returns whether the layers moved."""
        times = [None] * len(self.members)
        dist.all_gather_object(times, getattr(self.eng, "stage_s", 0.0))
        key = f"rebalance/{self.epoch}/{self.rebalances}"
        if self.root:
            S = getattr(self.eng, "S", getattr(self.eng, "n_stages", 1))
            per_stage = stage_s or [max(times[i] for i in range(len(times))
                                        if i // self.eng.tp == s) for s in range(S)]
            new = rebalancer.propose(self.eng.bounds, per_stage)
            self.store.set(key, ",".join(map(str, new)) if new else "")
        self.store.wait([key])
        val = self.store.get(key).decode()
        self.rebalances += 1
        if not val:
            return False
        bounds = [int(x) for x in val.split(",")]
        dist.barrier()
        self.eng = self.build_engine(bounds=bounds)
        return True

    def close(self):
        try:
            dist.destroy_process_group()
        except Exception:
            pass
