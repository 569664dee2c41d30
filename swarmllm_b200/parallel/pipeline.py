"""Pipeline parallelism: a model's layers cut into contiguous stages, one
stage per rank (one process per GPU, or per CPU process for the plumbing
config), activations passed stage to stage with point-to-point send/recv
(NCCL on GPUs, gloo on CPU).

The reference splits a model into layer ranges held by different peers and
forwards hidden states peer to peer per token
(src/inference/pipeline/distributed.rs:831,1054, wire format
src/network/protocol/layer_forward.rs:6), one request at a time.  Here:

* rank 0 owns the scheduler (continuous batching, chunked prefill) and the
  KV block manager; every stage keeps its own KV pages for its layers, indexed
  by the same slot ids, so one block table serves all stages;
* each engine step, rank 0 broadcasts the step plan (token rows, positions,
  slots, block tables) to all ranks and cuts the batch into micro-batches of
  whole sequences; every rank runs recv -> layers -> send per micro-batch, so
  stage r works on micro-batch m while stage r+1 works on m-1;
* the last stage selects tokens and sends them back to rank 0;
* activations cross as the fp32 residual stream, so a split run is
  bit-identical to a single-process run of the same batch (the two-CPU-peer tiny Llama setup).

Stage boundaries come from the native planner (`plan_bottleneck`) over
per-layer costs from the layout planner (parallel/planner.py): what each layer
reads per decode step, so attention / linear-attention / MoE layers weigh
what they cost.
"""
from __future__ import annotations

import itertools
import os
import time
from dataclasses import dataclass

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


def stage_bounds(n_layers: int, n_stages: int, extra_first: float = 0.0, extra_last: float = 0.0,
                 costs: list | None = None):
    """Layer boundaries [S+1] minimising the slowest stage.  `costs`: per-layer
    cost (parallel/planner.py layer_costs: what each layer reads per decode
    step, or measured timings); without it every layer costs 1 with the
    embedding and LM head folded into the first / last layer."""
    if costs is not None:
        from .planner import stage_plan
        return stage_plan(costs, [0.0] * n_layers, n_stages)[0]
    cost = [1.0] * n_layers
    cost[0] += extra_first
    cost[-1] += extra_last
    plan = native().plan_bottleneck(cost, [], [1.0] * n_stages, [], 0.0)
    if not plan.feasible:
        raise ValueError("cannot split %d layers into %d stages" % (n_layers, n_stages))
    return list(plan.first_layer)


@dataclass
class _MB:
    rows: slice          # token rows of this micro-batch in the step
    seqs: list           # batch indices of its sequences
    n_sample: int


class PipelineEngine:
    segments_served = 0    # layer-range forwards this rank ran (swarmllm_segments_served_total)
    bytes_sent = 0         # bytes this rank sent to other ranks (swarmllm_network_bytes_total)
    """Same API as LLMEngine (add_request / step / generate), run by every rank
    in lockstep; only rank 0 accepts requests and returns results."""

    def __init__(self, cfg: ModelConfig, ecfg: EngineConfig, source_factory, device,
                 group=None, micro_batches: int | None = None, use_graphs: bool = True,
                 tp: int = 1):
        """`tp` > 1: every stage is a tensor-parallel group of `tp` consecutive
        ranks (stage = rank // tp, lane = rank % tp); activations go from a
        lane of one stage to the same lane of the next."""
        self.cfg, self.ecfg = cfg, ecfg
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        assert self.world % tp == 0
        self.tp, self.lane = tp, self.rank % tp
        self.stage, self.n_stages = self.rank // tp, self.world // tp
        self.device = torch.device(device)
        self.gpu = self.device.type == "cuda"
        from .planner import layer_costs
        self.bounds = stage_bounds(cfg.n_layers, self.n_stages,
                                   costs=layer_costs(cfg, max(1, ecfg.max_running), 2048, tp))
        lo, hi = self.bounds[self.stage], self.bounds[self.stage + 1]
        self.lo, self.hi = lo, hi
        self.root = self.rank == 0  # owns the scheduler and the KV block manager
        self.first, self.last = self.stage == 0, self.stage == self.n_stages - 1
        self.micro = micro_batches or self.n_stages
        self.tpg = None
        if tp > 1:
            from .tp import TpGroup
            groups = [dist.new_group(list(range(s * tp, (s + 1) * tp)))
                      for s in range(self.n_stages)]
            self.tpg = TpGroup(self.lane, tp, device, groups[self.stage])
        src = source_factory()
        ps = ecfg.page_size
        self.max_pages = (ecfg.max_model_len + ps - 1) // ps
        pages = ecfg.kv_pages or ecfg.max_running * self.max_pages
        if self.gpu:
            from ..models.llama import LlamaGPU
            self.model = LlamaGPU(cfg, src, self.device, (lo, hi), tp=self.tpg)
            self.kv = PagedKVCache(hi - lo, pages + 1, self.model.n_kv, cfg.head_dim, self.device,
                                   ps)
            mt = ecfg.max_step_tokens
            self.ctx = self.model.make_context(mt, max(ecfg.max_running, 1), ecfg.max_model_len)
            self.sampler = DeviceSampler(self.device, max(ecfg.max_running, 1))
        else:
            from ..models.llama import LlamaCPU
            self.model = LlamaCPU(cfg, src, (lo, hi), native=ecfg.cpu_native)
            self.kv = PagedKVCache(hi - lo, pages + 1, cfg.n_kv_heads, cfg.head_dim, "cpu", ps,
                                   dtype=torch.float32)
            self.ctx = None
        self.trash_page = pages
        if self.root:
            N = native()
            self.bm = N.BlockManager(pages, ps, ecfg.prefix_cache)
            self.sched = N.Scheduler(self.bm, ecfg.max_step_tokens, ecfg.max_running,
                                     ecfg.prefill_chunk)
            self.params: dict[int, SamplingParams] = {}
            self._ids = itertools.count()
        self.use_graphs = use_graphs and self.gpu
        self.graphs: dict[int, tuple] = {}
        self.comm_dtype = torch.float32
        self.last_step_ms = 0.0
        self.record_logits: list | None = None  # last stage: keep every step's logits

    # ------------------------------------------------------------------ requests (rank 0)
    def add_request(self, prompt_ids, params: SamplingParams | None = None) -> int:
        assert self.root, "requests enter at rank 0"
        params = params or SamplingParams()
        rid = next(self._ids)
        eos = -1 if params.ignore_eos else params.eos_token_id
        self.sched.add_request(rid, [int(t) for t in prompt_ids], int(params.max_tokens), int(eos))
        self.params[rid] = params
        return rid

    def output(self, rid: int) -> list[int]:
        return [int(t) for t in self.sched.output(rid)]

    # ------------------------------------------------------------------ collectives
    def _bcast_plan(self, plan):
        """Rank 0 packs the step into one int32 tensor; everyone unpacks."""
        dev = self.device if self.gpu else torch.device("cpu")
        if self.root:
            tokens, positions, slots, bt_rows, seq_lens, sample_rows = plan_arrays(
                plan, self.bm, self.max_pages)
            N = len(tokens)
            B = len(plan.seq_ids)
            seq_start = np.asarray(plan.seq_start, np.int32)
            seq_ntok = np.asarray(plan.seq_ntok, np.int32)
            seq_samp = np.asarray(plan.seq_sample, np.int32)
            head = np.array([N, B, self.max_pages], np.int32)
            body = np.concatenate([tokens, positions, slots, seq_lens, seq_start, seq_ntok,
                                   seq_samp, bt_rows.reshape(-1)]).astype(np.int32)
            hdr = torch.from_numpy(head).to(dev)
        else:
            hdr = torch.zeros(3, dtype=torch.int32, device=dev)
        dist.broadcast(hdr, 0, group=self.group)
        N, B, mp = [int(v) for v in hdr.cpu()]
        size = 4 * N + 3 * B + N * mp
        buf = torch.from_numpy(body).to(dev) if self.root else torch.zeros(size, dtype=torch.int32, device=dev)
        if size:
            dist.broadcast(buf, 0, group=self.group)
        b = buf.cpu().numpy() if not self.root else body
        o = 0

        def take(n):
            nonlocal o
            r = b[o:o + n]
            o += n
            return r
        tokens, positions, slots, seq_lens = take(N), take(N), take(N), take(N)
        seq_start, seq_ntok, seq_samp = take(B), take(B), take(B)
        bt = take(N * mp).reshape(N, mp)
        return tokens, positions, slots, seq_lens, seq_start, seq_ntok, seq_samp, bt

    def _micro_batches(self, B, seq_start, seq_ntok, seq_samp):
        per = max(1, (B + self.micro - 1) // self.micro)
        out = []
        for i in range(0, B, per):
            seqs = list(range(i, min(B, i + per)))
            r0 = int(seq_start[seqs[0]])
            r1 = int(seq_start[seqs[-1]] + seq_ntok[seqs[-1]])
            out.append(_MB(slice(r0, r1), seqs, int(sum(seq_samp[s] for s in seqs))))
        return out

    # ------------------------------------------------------------------ step
    def step(self):
        plan = self.sched.schedule() if self.root else None
        tokens, positions, slots, seq_lens, seq_start, seq_ntok, seq_samp, bt = self._bcast_plan(plan)
        N, B = len(tokens), len(seq_start)
        if N == 0:
            return []
        mbs = self._micro_batches(B, seq_start, seq_ntok, seq_samp)
        dev = self.device if self.gpu else torch.device("cpu")
        sampled_all = []
        H = self.cfg.hidden
        pending = []
        for mb in mbs:
            r = mb.rows
            rows = r.stop - r.start
            samp_rows = np.array([int(seq_start[s] + seq_ntok[s] - 1) - r.start
                                  for s in mb.seqs if seq_samp[s]], np.int64)
            t = lambda a, dt=torch.int32: torch.as_tensor(np.ascontiguousarray(a), dtype=dt, device=dev)
            batch = StepBatch(t(tokens[r]), t(positions[r]), t(slots[r]), t(bt[r]), t(seq_lens[r]),
                              t(samp_rows, torch.int64), self.ecfg.max_model_len)
            if self.gpu:
                grp = attention_groups(None, self.cfg.n_heads // self.cfg.n_kv_heads,
                                       np.asarray(seq_start[mb.seqs]) - r.start,
                                       np.asarray(seq_ntok[mb.seqs]))
                if grp is not None:
                    batch.groups = (t(grp[0]), t(grp[1]), grp[2])
            h_in = None
            if not self.first:
                h_in = torch.empty(rows, H, dtype=self.comm_dtype, device=dev)
                dist.recv(h_in, self.rank - self.tp, group=self.group)
            out = self.model.forward(batch, self.kv, self.ctx, h_in)
            self.segments_served += 1
            if not self.last:
                # own buffer: the model's activation buffer is reused by the next micro-batch
                h = out.to(self.comm_dtype).clone()
                self.bytes_sent += h.numel() * h.element_size()
                req = dist.isend(h, self.rank + self.tp, group=self.group)
                pending.append((req, h))
            elif mb.n_sample and self.lane == 0:
                if self.record_logits is not None:
                    self.record_logits.append(out.detach().float().cpu().clone())
                params = self._params_for(mb.seqs, seq_samp)
                if self.gpu:
                    tok = self.sampler.sample(out, params, positions[r][samp_rows]).clone()
                else:
                    tok = torch.from_numpy(sample_host(out, params, positions[r][samp_rows]))
                sampled_all.append(tok.to(torch.int32))
        # Tokens go back to rank 0 in ONE message after the last micro-batch: with
        # 2 ranks the pair (0, 1) carries both directions in one ordered NCCL
        # stream, and per-micro-batch token sends would wait on activation sends.
        n_samp_total = sum(mb.n_sample for mb in mbs)
        last_lane0 = (self.n_stages - 1) * self.tp  # global rank that samples
        if self.last and self.lane == 0 and not self.root and n_samp_total:
            toks = torch.cat(sampled_all).contiguous()
            self.bytes_sent += toks.numel() * toks.element_size()
            dist.send(toks, 0, group=self.group)
        for req, _ in pending:
            req.wait()
        if self.root:
            if last_lane0 != 0:
                sampled = np.zeros(0, np.int32)
                if n_samp_total:
                    tok = torch.empty(n_samp_total, dtype=torch.int32, device=dev)
                    dist.recv(tok, last_lane0, group=self.group)
                    sampled = tok.cpu().numpy()
            else:
                sampled = (torch.cat(sampled_all).cpu().numpy() if sampled_all
                           else np.zeros(0, np.int32))
            done = set(int(d) for d in self.sched.commit(plan, sampled.tolist()))
            out = []
            k = 0
            for sid, s in zip(plan.seq_ids, plan.seq_sample):
                if s:
                    out.append((int(sid), int(sampled[k]), int(sid) in done))
                    k += 1
            return out
        return []

    def _params_for(self, seqs, seq_samp):
        # Sampling parameters live on rank 0; the last stage uses greedy unless
        # the run passes parameters to every rank (generate() does).
        ps = getattr(self, "_step_params", None)
        if ps is None:
            return [SamplingParams() for s in seqs if seq_samp[s]]
        return [ps[s] for s in seqs if seq_samp[s]]

    def has_work(self) -> bool:
        flag = torch.tensor([1 if (self.root and self.sched.has_work()) else 0], dtype=torch.int32,
                            device=self.device if self.gpu else "cpu")
        dist.broadcast(flag, 0, group=self.group)
        return bool(flag.item())

    def generate(self, prompts, params: SamplingParams | None = None):
        """Collective: every rank calls it with the same prompts; rank 0 returns
        the generated tokens (other ranks return None)."""
        params = params or SamplingParams()
        res = {}
        if self.root:
            rids = [self.add_request(p, params) for p in prompts]
            res = {r: [] for r in rids}
        while self.has_work():
            for rid, tok, fin in self.step():
                res[rid].append(tok)
        if self.root:
            return [res[r] for r in sorted(res)]
        return None


def init_distributed(backend: str | None = None, timeout_s: float = 120.0):
    """Initialise torch.distributed from torchrun env vars (127.0.0.1)."""
    import datetime
    if dist.is_initialized():
        return
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    backend = backend or ("nccl" if torch.cuda.is_available() else "gloo")
    kw = {}
    if backend == "nccl":
        lr = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(lr)
        kw["device_id"] = torch.device(f"cuda:{lr}")
    dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
