"""Tensor-parallel serving engine: one model split over the W GPUs of a group,
the whole decode step captured in a CUDA graph on every rank.

    eng = TpEngine.create(cfg, ecfg, source_factory)      # collective, every rank
    if eng.root:
        outs = eng.generate(prompts, params)              # drives every rank
        eng.stop()
    else:
        eng.follow()                                       # until the root stops

Rank 0 owns the scheduler (continuous batching, chunked prefill), the KV
block manager and the sampling; it is an ordinary LLMEngine whose runner
sends every step's plan (token rows, positions, KV slots, block tables, the
graph-or-eager decision) to the other ranks over a CPU (gloo) group before it
runs the step itself.  The other ranks replay the same CUDA graph (or run the
same eager forward) on their shards.  GPUs meet only inside the fused
kernels: the row-parallel GEMMs push their owner-routed partials over NVLink
and tp_reduce_norm all-gathers the residual stream (parallel/tp.py), so a
step costs one plan message on the host and no collective call on the GPU.

Every rank builds the same graphs in the same order (capture warms each size
up with two forwards, which already exchange data between the ranks), and
the KV page count is the minimum over the ranks, so the root's page ids are
valid everywhere.

Reference behaviour: the reference runs a tensor-parallel segment by sending
each layer's phases to its peers and all-reducing per phase over the network
(src/inference/pipeline/tensor_parallel.rs:20, split/executor.rs:3471).
"""
from __future__ import annotations

import datetime
import os

import numpy as np
import torch
import torch.distributed as dist

from ..engine.engine import EngineConfig, LLMEngine
from ..engine.sampling import SamplingParams
from ..models.config import ModelConfig

_STOP, _STEP, _REPLAY = 0, 1, 2
_HDR = 8  # int64 header: kind, N, B, max_pages, n_prefill, use_graph, replay size, replay count


class _PlanView:
    """A StepPlan rebuilt from the root's message (what GpuRunner.run reads)."""

    def __init__(self, tokens, positions, slots, row_seq, seq_ids, seq_start, seq_ntok,
                 seq_sample, n_prefill):
        self.tokens, self.positions, self.slots = tokens, positions, slots
        self.row_seq, self.seq_ids = row_seq, seq_ids
        self.seq_start, self.seq_ntok, self.seq_sample = seq_start, seq_ntok, seq_sample
        self.n_prefill_tokens = n_prefill

    def __len__(self):
        return len(self.tokens)


class _TablesView:
    """Block tables of the plan's sequences, as the root's block manager gave them."""

    def __init__(self, bt_seq: np.ndarray):
        self.bt = bt_seq

    def block_table(self, seq_ids, max_pages):
        return self.bt


class _BroadcastingRunner:
    """The root's runner: sends the step to the other ranks, then runs it.
    Recurrent-state slots the root frees (hybrid models) travel with the next
    step, so every rank keeps the same slot table."""

    def __init__(self, eng: "TpEngine", inner):
        self._eng, self._inner = eng, inner
        self.released: list[int] = []
        if inner.slots is not None:
            real = inner.slots.release

            def release(sid):
                if sid in inner.slots.of:
                    self.released.append(int(sid))
                real(sid)
            inner.slots.release = release

    def __getattr__(self, name):
        return getattr(self._inner, name)

    def run(self, plan, block_manager, params, history=None):
        r = self._inner
        use_graph = all(p.greedy and not p.penalized for p in params)
        ids = [int(s) for s in plan.seq_ids]
        bt_seq = (block_manager.block_table(ids, r.max_pages) if ids
                  else np.zeros((0, r.max_pages), np.int32))
        self._eng._send_step(plan, bt_seq, use_graph)
        return r.run(plan, block_manager, params, history)


class TpEngine(LLMEngine):
    @classmethod
    def create(cls, cfg: ModelConfig, ecfg: EngineConfig, source_factory, device=None,
               timeout_s: float = 120.0) -> "TpEngine":
        """Collective over the default process group (NCCL, one rank per GPU):
        every rank holds 1/W of every layer."""
        from ..models.llama import LlamaGPU
        from .tp import TpGroup
        rank, world = dist.get_rank(), dist.get_world_size()
        dev = torch.device(device or f"cuda:{int(os.environ.get('LOCAL_RANK', rank))}")
        torch.cuda.set_device(dev)
        tpg = TpGroup(rank, world, dev, None)
        cpu = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=timeout_s))
        model = LlamaGPU(cfg, source_factory(), dev, tp=tpg)
        ecfg = EngineConfig(**{**ecfg.__dict__})
        if model.n_lin_layers:
            # saved recurrent states (hybrid prefix hits) are copied on the root only
            ecfg.prefix_cache = False
        if not ecfg.kv_pages:  # the same page count everywhere: the minimum over the ranks
            free, _ = torch.cuda.mem_get_info(dev)
            from ..ops.attention import PagedKVCache
            per_page = PagedKVCache.bytes_per_page(model.n_kv_layers, model.n_kv, cfg.head_dim,
                                                   ecfg.page_size)
            budget = free * ecfg.kv_fraction - 4 * (1 << 30)
            need = ecfg.max_running * ((ecfg.max_model_len + ecfg.page_size - 1) // ecfg.page_size)
            pages = torch.tensor([int(max(64, min(budget // per_page, need)))], dtype=torch.int64)
            dist.all_reduce(pages, op=dist.ReduceOp.MIN, group=cpu)
            ecfg.kv_pages = int(pages.item())
        eng = cls(model, cfg, ecfg, dev)
        eng.tpg, eng.cpu_group = tpg, cpu
        eng.rank, eng.world = rank, world
        eng.root = rank == 0
        if eng.root:
            eng.runner = _BroadcastingRunner(eng, eng.runner)
        return eng

    # ------------------------------------------------------------------ messages
    def _bcast(self, t: torch.Tensor):
        dist.broadcast(t, 0, group=self.cpu_group)

    def _send_step(self, plan, bt_seq: np.ndarray, use_graph: bool):
        N, B = len(plan.tokens), len(plan.seq_ids)
        mp = self.runner._inner.max_pages
        rel = self.runner.released
        self.runner.released = []
        hdr = torch.tensor([_STEP, N, B, mp, int(plan.n_prefill_tokens), int(use_graph), len(rel), 0],
                           dtype=torch.int64)
        self._bcast(hdr)
        body = np.concatenate([np.asarray(a, np.int64).reshape(-1) for a in (
            plan.tokens, plan.positions, plan.slots, plan.row_seq, plan.seq_ids, plan.seq_start,
            plan.seq_ntok, plan.seq_sample, bt_seq, rel)])
        self._bcast(torch.from_numpy(np.ascontiguousarray(body, dtype=np.int32)))

    def stop(self):
        """Root: release the followers (they return from follow())."""
        assert self.root
        self._bcast(torch.zeros(_HDR, dtype=torch.int64))

    def replay(self, batch: int, count: int, events=None):
        """Collective timing hook: every rank replays its captured decode graph
        of `batch` rows `count` times (inputs as left by the last step).  The
        root calls it; followers run it from follow().  `events`: a (start,
        end) CUDA-event pair recorded around the replays on this rank."""
        if self.root:
            self._bcast(torch.tensor([_REPLAY, 0, 0, 0, 0, 1, batch, count], dtype=torch.int64))
        runner = self.runner._inner if self.root else self.runner
        g = runner.graphs[batch][0]
        if events is not None:
            events[0].record()
        for _ in range(count):
            g.replay()
        if events is not None:
            events[1].record()
        self.last_replay_events = events

    def follow(self, on_replay=None):
        """Followers: run the root's steps until it stops.  `on_replay(ms)`
        receives each timed replay's device time on this rank."""
        assert not self.root
        runner = self.runner
        while True:
            hdr = torch.zeros(_HDR, dtype=torch.int64)
            self._bcast(hdr)
            kind, N, B, mp, n_pf, use_graph, rb, rc = (int(v) for v in hdr)
            if kind == _STOP:
                return
            if kind == _REPLAY:
                ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                self.replay(rb, rc, ev)
                if on_replay is not None:
                    torch.cuda.synchronize(self.device)
                    on_replay(ev[0].elapsed_time(ev[1]))
                continue
            n_rel = rb    # header slot 6: recurrent-state slots the root released
            body = torch.zeros(4 * N + 4 * B + B * mp + n_rel, dtype=torch.int32)
            self._bcast(body)
            b = body.numpy()
            o = 0

            def take(n):
                nonlocal o
                r = b[o:o + n]
                o += n
                return r
            tokens, positions, slots, row_seq = take(N), take(N), take(N), take(N)
            seq_ids, seq_start, seq_ntok, seq_samp = take(B), take(B), take(B), take(B)
            bt_seq = take(B * mp).reshape(B, mp)
            if n_rel and runner.slots is not None:
                for sid in take(n_rel).tolist():
                    runner.slots.release(int(sid))
            plan = _PlanView(tokens, positions, slots, row_seq, seq_ids, seq_start, seq_ntok,
                             seq_samp, n_pf)
            n_samp = int(np.sum(seq_samp))
            params = [SamplingParams(temperature=0.0 if use_graph else 1.0)] * n_samp
            runner.run(plan, _TablesView(bt_seq), params)
            self.steps += 1

    def close(self):
        """Collective teardown of the peer mappings."""
        self.runner = getattr(self.runner, "_inner", self.runner)
        self.runner.graphs.clear()
        torch.cuda.synchronize(self.device)
        self.tpg.close()
