"""Pipeline parallelism without per-step bubbles: independent waves.

The synchronous PipelineEngine runs one global step at a time: S micro-batches
through S stages fill and drain the pipeline every step (S / (2S - 1) of the
stage time is useful).  Here the running sequences are split into V waves,
each with its own scheduler and block manager over a disjoint range of the KV
pages.  A wave's step -- its plan plus its activations -- travels stage to
stage by point-to-point sends; the root schedules a wave's next step as soon
as that wave's sampled tokens come back from the last stage.  With V = S waves
every stage always has a wave to work on, and each wave step still reads a
stage's weights once for the whole wave's batch.

Messages between neighbouring stages (same TP lane), in issue order:
  header int32[8] = (kind, wave, N rows, B seqs, max_pages, n_sample, 0, 0)
  plan   int32[4N + 3B + N*max_pages]  (tokens, positions, slots, lens,
         seq_start, seq_ntok, seq_sample, block-table rows)
  hidden fp32 [N, hidden]                (not sent into stage 0)
The last stage's lane 0 returns the sampled token ids to the root.  kind 2
= stop.  All sends are non-blocking, so the root sending a wave onward while
the last stage returns another wave's tokens cannot deadlock.  Inside a
stage's tensor-parallel group, stage 0 lanes get the header and plan by a
broadcast from the root; other stages' lanes receive them from the previous
stage's same lane.

A long prompt is prefilled in chunks (the scheduler's prefill_chunk); a chunk
that samples nothing is committed as soon as it is sent, so the wave's next
chunk follows it down the chain and up to one chunk per stage is in flight:
the stages prefill one prompt together instead of in turn.

Reference: the reference pipelines a prompt's chunks through every segment
at once (pipeline/prompt_chunks.rs) and keeps several requests in flight on a
split model; one request's tokens still go one at a time through the chain.
"""
from __future__ import annotations

import itertools
import time
from collections import deque

import numpy as np
import torch
import torch.distributed as dist

from ..engine.engine import EngineConfig
from ..engine.runner import attention_groups, plan_arrays
from ..engine.sampling import DeviceSampler, SamplingParams, sample_host
from ..models.config import ModelConfig
from ..models.llama import StepBatch
from ..ops.attention import PagedKVCache
from ..utils.ext import native
from .pipeline import stage_bounds

_STEP, _STOP = 1, 2


class AsyncPipelineEngine:
    segments_served = 0    # layer-range forwards this rank ran (swarmllm_segments_served_total)
    bytes_sent = 0         # bytes this rank sent to other ranks (swarmllm_network_bytes_total)
    def __init__(self, cfg: ModelConfig, ecfg: EngineConfig, source_factory, device,
                 tp: int = 1, waves: int | None = None, bounds: list | None = None):
        """`bounds`: layer boundaries [stages + 1] (default: the layout planner's
        cut over its per-layer costs; the rebalancer passes measured ones)."""
        self.cfg, self.ecfg = cfg, ecfg
        self.rank, self.world = dist.get_rank(), dist.get_world_size()
        assert self.world % tp == 0
        self.tp, self.lane = tp, self.rank % tp
        self.stage, self.S = self.rank // tp, self.world // tp
        self.device = torch.device(device)
        self.gpu = self.device.type == "cuda"
        from .planner import layer_costs
        self.bounds = list(bounds) if bounds is not None else stage_bounds(
            cfg.n_layers, self.S, costs=layer_costs(cfg, max(1, ecfg.max_running), 2048, tp))
        assert len(self.bounds) == self.S + 1 and self.bounds[-1] == cfg.n_layers
        lo, hi = self.bounds[self.stage], self.bounds[self.stage + 1]
        self.lo, self.hi = lo, hi
        self.root = self.rank == 0
        self.first, self.last = self.stage == 0, self.stage == self.S - 1
        self.V = waves or self.S
        self.prev = self.rank - tp if not self.first else None
        self.next = self.rank + tp if not self.last else None
        self.sampler_rank = (self.S - 1) * tp
        self.tpg = self.stage_group = None
        if tp > 1:
            from .tp import TpGroup
            groups = [dist.new_group(list(range(s * tp, (s + 1) * tp))) for s in range(self.S)]
            self.stage_group = groups[self.stage]
            self.tpg = TpGroup(self.lane, tp, device, self.stage_group)
        src = source_factory()
        ps = ecfg.page_size
        self.max_pages = (ecfg.max_model_len + ps - 1) // ps
        per_wave_running = max(1, (ecfg.max_running + self.V - 1) // self.V)
        self.pages_per_wave = ecfg.kv_pages // self.V if ecfg.kv_pages else \
            per_wave_running * self.max_pages
        pages = self.pages_per_wave * self.V
        if self.gpu:
            from ..models.llama import LlamaGPU
            self.model = LlamaGPU(cfg, src, self.device, (lo, hi), tp=self.tpg)
            self.kv = PagedKVCache(hi - lo, pages + 1, self.model.n_kv, cfg.head_dim,
                                   self.device, ps)
            self.ctx = self.model.make_context(ecfg.max_step_tokens, per_wave_running,
                                               ecfg.max_model_len)
            self.sampler = DeviceSampler(self.device, per_wave_running)
        else:
            from ..models.llama import LlamaCPU
            self.model = LlamaCPU(cfg, src, (lo, hi), native=ecfg.cpu_native)
            self.kv = PagedKVCache(hi - lo, pages + 1, cfg.n_kv_heads, cfg.head_dim, "cpu", ps,
                                   dtype=torch.float32)
            self.ctx = None
        if self.root:
            N = native()
            self.bms = [N.BlockManager(self.pages_per_wave, ps, ecfg.prefix_cache)
                        for _ in range(self.V)]
            self.scheds = [N.Scheduler(self.bms[v], ecfg.max_step_tokens, per_wave_running,
                                       ecfg.prefill_chunk) for v in range(self.V)]
            self.params: dict[int, SamplingParams] = {}
            self.wave_of: dict[int, int] = {}
            self._ids = itertools.count()
        self.comm_dev = self.device if self.gpu else torch.device("cpu")
        self._pending = deque()
        self.stage_s = 0.0  # moving average of this stage's forward time (rebalancer)
        self.retired = 0  # wave steps completed (root)
        self.chunks_pipelined = 0  # prompt chunks sent behind another of their wave (root)

    # ------------------------------------------------------------------ requests (root)
    def add_request(self, prompt_ids, params: SamplingParams | None = None) -> int:
        assert self.root, "requests enter at rank 0"
        params = params or SamplingParams()
        rid = next(self._ids)
        v = min(range(self.V), key=lambda w: sum(1 for r, x in self.wave_of.items() if x == w
                                                   and not self.scheds[w].finished(r)))
        eos = -1 if params.ignore_eos else params.eos_token_id
        self.scheds[v].add_request(rid, [int(t) for t in prompt_ids], int(params.max_tokens),
                                   int(eos))
        self.params[rid] = params
        self.wave_of[rid] = v
        return rid

    def output(self, rid: int) -> list[int]:
        return [int(t) for t in self.scheds[self.wave_of[rid]].output(rid)]

    def release(self, rid: int):
        v = self.wave_of.pop(rid)
        self.scheds[v].release(rid)
        self.params.pop(rid, None)

    def abort(self, rid: int):
        self.scheds[self.wave_of[rid]].abort(rid)

    # ------------------------------------------------------------------ plumbing
    def _isend(self, t: torch.Tensor, dst: int):
        self.bytes_sent += t.numel() * t.element_size()
        self._pending.append((dist.isend(t, dst), t))
        while len(self._pending) > 8:
            req, _ = self._pending.popleft()
            req.wait()

    def _flush(self):
        while self._pending:
            req, _ = self._pending.popleft()
            req.wait()

    def _pack(self, v: int, plan):
        off_pages = v * self.pages_per_wave
        tokens, positions, slots, bt, lens, _ = plan_arrays(plan, self.bms[v], self.max_pages)
        ps = self.ecfg.page_size
        slots = np.asarray(slots, np.int64) + off_pages * ps
        bt = np.asarray(bt, np.int64) + off_pages
        N, B = len(tokens), len(plan.seq_ids)
        samp = np.asarray(plan.seq_sample, np.int32)
        hdr = np.array([_STEP, v, N, B, self.max_pages, int(samp.sum()), 0, 0], np.int32)
        body = np.concatenate([tokens, positions, slots, lens, plan.seq_start, plan.seq_ntok, samp,
                               bt.reshape(-1)]).astype(np.int32)
        return hdr, body

    def _unpack(self, hdr, body):
        N, B, mp = int(hdr[2]), int(hdr[3]), int(hdr[4])
        o = 0

        def take(n):
            nonlocal o
            r = body[o:o + n]
            o += n
            return r
        tokens, positions, slots, lens = take(N), take(N), take(N), take(N)
        seq_start, seq_ntok, seq_samp = take(B), take(B), take(B)
        bt = take(N * mp).reshape(N, mp)
        return tokens, positions, slots, lens, seq_start, seq_ntok, seq_samp, bt

    def _forward(self, hdr, body, h_in):
        tokens, positions, slots, lens, seq_start, seq_ntok, seq_samp, bt = self._unpack(hdr, body)
        samp_rows = np.array([int(seq_start[s] + seq_ntok[s] - 1) for s in range(len(seq_start))
                              if seq_samp[s]], np.int64)
        d = self.comm_dev
        t = lambda a, dt=torch.int32: torch.as_tensor(np.ascontiguousarray(a), dtype=dt, device=d)
        batch = StepBatch(t(tokens), t(positions), t(slots), t(bt), t(lens),
                          t(samp_rows, torch.int64), self.ecfg.max_model_len)
        if self.gpu:  # prefill chunks: multi-position row groups on the tensor-core attention
            grp = attention_groups(None, self.cfg.n_heads // self.cfg.n_kv_heads, seq_start, seq_ntok)
            if grp is not None:
                batch.groups = (t(grp[0]), t(grp[1]), grp[2])
        t0 = time.perf_counter()
        out = self.model.forward(batch, self.kv, self.ctx, h_in)
        if self.gpu:
            torch.cuda.current_stream(self.device).synchronize()
        self.stage_s = 0.8 * self.stage_s + 0.2 * (time.perf_counter() - t0) \
            if self.stage_s else time.perf_counter() - t0
        self.segments_served += 1
        return out, positions[samp_rows] if len(samp_rows) else positions[:0]

    def _recv_msg(self, src: int):
        d = self.comm_dev
        hdr = torch.empty(8, dtype=torch.int32, device=d)
        dist.recv(hdr, src)
        h = hdr.cpu().numpy()
        if h[0] == _STOP:
            return h, None, None
        N, B, mp = int(h[2]), int(h[3]), int(h[4])
        body = torch.empty(4 * N + 3 * B + N * mp, dtype=torch.int32, device=d)
        dist.recv(body, src)
        hid = torch.empty(N, self.cfg.hidden, dtype=torch.float32, device=d)
        dist.recv(hid, src)
        return h, body.cpu().numpy(), hid

    def _tp_bcast(self, hdr: np.ndarray | None, body: np.ndarray | None):
        """Stage 0 lanes: the root's header and plan go to the other lanes."""
        d = self.comm_dev
        src = 0
        h = torch.from_numpy(hdr).to(d) if self.lane == 0 else torch.empty(8, dtype=torch.int32, device=d)
        dist.broadcast(h, src, group=self.stage_group)
        hn = h.cpu().numpy()
        if hn[0] == _STOP:
            return hn, None
        N, B, mp = int(hn[2]), int(hn[3]), int(hn[4])
        b = torch.from_numpy(body).to(d) if self.lane == 0 else \
            torch.empty(4 * N + 3 * B + N * mp, dtype=torch.int32, device=d)
        dist.broadcast(b, src, group=self.stage_group)
        return hn, b.cpu().numpy()

    def _stage_step(self, hdr, body, h_in):
        """Forward one wave step here and pass it on (or sample and return it)."""
        out, pos = self._forward(hdr, body, h_in)
        if not self.last:
            d = self.comm_dev
            self._isend(torch.from_numpy(hdr).to(d), self.next)
            self._isend(torch.from_numpy(body).to(d), self.next)
            self._isend(out.to(torch.float32).clone(), self.next)
            return None
        if self.lane != 0:
            return None
        n_samp = int(hdr[5])
        if n_samp == 0:  # nothing to return: the root posts no receive for this step
            return np.zeros(0, np.int32) if self.root else None
        else:
            params = [SamplingParams()] * n_samp  # greedy on the last stage
            if self.gpu:
                tok = self.sampler.sample(out, params, pos).to(torch.int32).clone()
            else:
                tok = torch.from_numpy(sample_host(out, params, pos)).to(torch.int32)
        if self.root:
            return tok.cpu().numpy()
        self._isend(tok, 0)
        return None

    # ------------------------------------------------------------------ root loop
    def _root_round(self, inflight: deque, busy: list, issue: bool = True) -> list:
        """Issue every idle wave that has work (unless draining), then retire
        the oldest wave in flight.  Returns (request id, token, finished) events."""
        events = []
        for v in range(self.V):
            chunks = 0
            while issue and not busy[v] and self.scheds[v].has_work() and chunks < self.S:
                plan = self.scheds[v].schedule()
                if len(plan) == 0:
                    break
                hdr, body = self._pack(v, plan)
                if self.tp > 1:
                    self._tp_bcast(hdr, body)
                res = self._stage_step(hdr, body, None)
                if int(np.sum(plan.seq_sample)) == 0:
                    # A prompt chunk that samples nothing returns nothing: commit it
                    # now and send the wave's next chunk right behind it, so a long
                    # prompt's chunks fill the stages at once (up to one per stage).
                    self.scheds[v].commit(plan, [])
                    self.chunks_pipelined += 1
                    chunks += 1
                    continue
                busy[v] = True
                inflight.append((v, plan, res))
        if not inflight:
            return events
        v, plan, res = inflight.popleft()
        n_samp = int(np.sum(plan.seq_sample))
        if res is None:  # another rank samples
            tok = torch.empty(n_samp, dtype=torch.int32, device=self.comm_dev)
            if n_samp:
                dist.recv(tok, self.sampler_rank)
            res = tok.cpu().numpy()
        done = set(int(x) for x in self.scheds[v].commit(plan, res.tolist()))
        k = 0
        for sid, s in zip(plan.seq_ids, plan.seq_sample):
            if s:
                events.append((int(sid), int(res[k]), int(sid) in done))
                k += 1
        busy[v] = False
        self.retired += 1
        return events

    def _stop(self):
        hdr = np.array([_STOP, 0, 0, 0, 0, 0, 0, 0], np.int32)
        if self.tp > 1:
            self._tp_bcast(hdr, None)
        if self.next is not None:
            self._isend(torch.from_numpy(hdr).to(self.comm_dev), self.next)
        self._flush()

    # ------------------------------------------------------------------ collective API
    def run(self, on_events=None, stop_when=None, on_step=None):
        """Collective: every rank calls it.  The root drives until no wave has
        work (or `stop_when()` is true) and passes events to on_events.
        `on_step()` runs on every rank after each wave step it handled (the
        failover layer heartbeats there; an exception it raises ends run)."""
        if self.root:
            inflight, busy = deque(), [False] * self.V
            draining = False
            while True:
                if not draining and stop_when is not None and stop_when():
                    draining = True  # issue nothing more; retire what is in flight
                ev = self._root_round(inflight, busy, issue=not draining)
                if on_events and ev:
                    on_events(ev)
                if on_step is not None:
                    on_step()
                if not inflight and (draining or not any(s.has_work() for s in self.scheds)):
                    break
            self._stop()
            return
        while True:
            if self.first:  # stage-0 lanes of a TP group
                hdr, body = self._tp_bcast(None, None)
                h_in = None
            else:
                hdr, body, h_in = self._recv_msg(self.prev)
            if hdr[0] == _STOP:
                if self.next is not None:
                    self._isend(torch.from_numpy(hdr).to(self.comm_dev), self.next)
                self._flush()
                return
            self._stage_step(hdr, body, h_in)
            if on_step is not None:
                on_step()

    def generate(self, prompts, params: SamplingParams | None = None):
        """Collective; the root returns the generated tokens per prompt."""
        res = {}
        if self.root:
            rids = [self.add_request(p, params) for p in prompts]
            res = {r: [] for r in rids}

        def take(ev):
            for rid, tok, _ in ev:
                res[rid].append(tok)
        self.run(on_events=take)
        if self.root:
            out = [res[r] for r in sorted(res)]
            for r in list(res):
                self.release(r)
            return out
        return None
