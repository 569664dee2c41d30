"""LLMEngine: the public single-process inference API.

    eng = LLMEngine.from_config(preset("llama-3.2-3b"), device="cuda:0")
    outs = eng.generate([[1, 2, 3]], SamplingParams(max_tokens=32))

One engine owns: the C++ BlockManager (paged KV pages + prefix cache), the
C++ Scheduler (continuous batching, chunked prefill, preemption), a runner
(GPU with CUDA graphs, or CPU) and per-request sampling parameters.  Each
``step()`` = schedule -> one forward over the mixed batch -> token selection
-> commit.  Finished requests are reported with their tokens and timings.
Reference: the worker's run loop (src/inference/model_worker.rs:173,11934)
plus ModelProcessPool::generate (src/inference/process_pool.rs:14208).
"""
from __future__ import annotations

import collections
import dataclasses
import hashlib
import itertools
import time
from dataclasses import dataclass

import numpy as np
import torch

from ..models.config import ModelConfig
from ..ops.attention import PagedKVCache
from ..utils.ext import native
from ..utils.tracing import RequestTrace, StageProfiler
from .runner import CpuRunner, GpuRunner
from .sampling import SamplingParams


RECENT_PROMPTS = 256   # released base-model prompts remembered for persisting the prefix cache


def cache_salt(lora: str | None) -> int:
    """Root of a request's prefix-cache hash chain: 0 for the base model, a
    64-bit digest of the adapter name under a LoRA adapter, so the KV pages of
    different adapters are never shared."""
    if lora is None:
        return 0
    return int.from_bytes(hashlib.blake2b(lora.encode(), digest_size=8).digest(), "little") | 1


@dataclass
class EngineConfig:
    max_model_len: int = 4096
    max_step_tokens: int = 2048     # per-step token budget (prefill chunk + decodes)
    max_running: int = 64           # max concurrent sequences
    prefill_chunk: int = 2048       # reference default is 128 (config/default.toml); B200 affords more
    page_size: int = 16
    kv_pages: int = 0               # 0 -> derive from kv_fraction of free memory
    kv_fraction: float = 0.85       # reference VRAM_HEADROOM_PCT = 85 (split/kv_budget.rs:58)
    prefix_cache: bool = True
    cuda_graphs: bool = True
    graph_sizes: tuple = (1, 2, 4, 8, 16, 32, 64)
    max_loras: int = 0              # LoRA adapter slots (0: LoRA off)
    state_cache_entries: int = 8    # hybrid models: saved recurrent states for prefix hits
    max_lora_rank: int = 64
    # speculative serving (engine/spec_engine.py): a drafter preset name, "self"
    # (the target drafts for itself) or "ngram" (prompt lookup); "" = off
    draft_model: str = ""
    spec_depth: int = 4
    spec_width: int = 4
    # CPU device only: dense Q4_K/Q6_K/Q8_0 projections stay quantized and run
    # through the native int8-dot matmul, attention through the native kernel
    cpu_native: bool = False


@dataclass
class RequestOutput:
    request_id: int
    prompt_len: int
    token_ids: list
    finished: bool
    trace: RequestTrace | None = None


class LLMEngine:
    def __init__(self, model, cfg: ModelConfig, ecfg: EngineConfig, device="cuda:0"):
        self.cfg, self.ecfg = cfg, ecfg
        self.device = torch.device(device)
        self.model = model
        N = native()
        ps = ecfg.page_size
        lin = model.linear_state_spec() if hasattr(model, "linear_state_spec") else None
        if lin is not None and ecfg.state_cache_entries <= 0:
            # recurrent state cannot be rebuilt from cached KV pages alone
            ecfg.prefix_cache = False
        n_kv_layers = getattr(model, "n_kv_layers", model.hi - model.lo)
        self.lora_of: dict[int, int] = {}
        self.lora_names: list[str] = []
        self.images: dict[int, list] = {}   # request id -> [(first position, image rows)]
        self.vision = None
        if ecfg.max_loras and self.device.type == "cuda":
            model.enable_lora(ecfg.max_loras, ecfg.max_lora_rank)
        elif ecfg.max_loras:
            model.lora_adapters = []
        if self.device.type == "cuda":
            pages = ecfg.kv_pages or self._auto_pages()
            # one extra page: the trash page that graph padding rows write to
            self.kv = PagedKVCache(n_kv_layers, pages + 1, getattr(model, "n_kv", cfg.n_kv_heads),
                                   cfg.head_dim, self.device, ps)
            if lin is not None:
                self.kv.add_linear_state(lin[0], max(ecfg.max_running, max(ecfg.graph_sizes)) + 1,
                                         *lin[1:])
            self.bm = N.BlockManager(pages, ps, ecfg.prefix_cache)
            self.runner = GpuRunner(model, self.kv, ecfg.max_step_tokens, ecfg.max_running,
                                    ecfg.max_model_len, ecfg.graph_sizes, ecfg.cuda_graphs,
                                    trash_page=pages)
            self.runner.lora_of = self.lora_of if ecfg.max_loras else None
            self.runner.images = self.images
            if ecfg.cuda_graphs:
                self.runner.capture_graphs()
        else:
            pages = ecfg.kv_pages or (ecfg.max_running * ((ecfg.max_model_len + ps - 1) // ps))
            self.kv = PagedKVCache(n_kv_layers, pages, cfg.n_kv_heads, cfg.head_dim, "cpu", ps,
                                   dtype=torch.float32)
            if lin is not None:
                self.kv.add_linear_state(lin[0], ecfg.max_running + 1, *lin[1:])
            self.bm = N.BlockManager(pages, ps, ecfg.prefix_cache)
            self.runner = CpuRunner(model, self.kv, ecfg.max_model_len, ecfg.max_running)
            self.runner.lora_of = self.lora_of if ecfg.max_loras else None
            self.runner.images = self.images
        self.sched = N.Scheduler(self.bm, ecfg.max_step_tokens, ecfg.max_running, ecfg.prefill_chunk)
        self.state_cache = None
        self._hyb: dict[int, dict] = {}     # hybrid requests: pending state restore / save
        self._gen_counts: dict[int, collections.Counter] = {}  # penalized requests' outputs
        if lin is not None and ecfg.prefix_cache:
            from .state_cache import StateCache
            self.state_cache = StateCache(self.kv, ecfg.state_cache_entries)
        self.params: dict[int, SamplingParams] = {}
        self.traces: dict[int, RequestTrace] = {}
        self.prompt_len: dict[int, int] = {}
        self._prompts: dict[int, np.ndarray] = {}   # base-model prompts in flight
        self._recent: collections.OrderedDict = collections.OrderedDict()  # released, LRU
        self._ids = itertools.count()
        self.profiler = StageProfiler()
        model.profiler = self.profiler     # per-stage accounting inside the forward
        self.steps = 0

    # ------------------------------------------------------------------ construction
    @classmethod
    def from_config(cls, cfg: ModelConfig, device="cuda:0", ecfg: EngineConfig | None = None,
                    source=None, seed: int = 0, ep=None, tp=None):
        """`ep`: expert-parallel group (parallel/ep.py) for MoE models served
        with the experts split over the GPUs of a node."""
        from ..models.llama import LlamaCPU, LlamaGPU
        from ..models.weights import RandomSource
        ecfg = ecfg or EngineConfig()
        dev = torch.device(device)
        if source is None:
            source = RandomSource(cfg, seed=seed, on_device=dev.type == "cuda")
        if dev.type == "cuda":
            model = LlamaGPU(cfg, source, dev, ep=ep, tp=tp)
        else:
            model = LlamaCPU(cfg, source, native=ecfg.cpu_native)
        return cls(model, cfg, ecfg, dev)

    @classmethod
    def from_gguf(cls, path: str, device="cuda:0", ecfg: EngineConfig | None = None):
        from ..models.weights import GgufSource
        src = GgufSource(path)
        eng = cls.from_config(src.cfg, device, ecfg, source=src)
        eng.source_path = path
        return eng

    def _auto_pages(self) -> int:
        free, _ = torch.cuda.mem_get_info(self.device)
        per_page = PagedKVCache.bytes_per_page(getattr(self.model, "n_kv_layers",
                                                       self.model.hi - self.model.lo),
                                               getattr(self.model, "n_kv", self.cfg.n_kv_heads),
                                               self.cfg.head_dim, self.ecfg.page_size)
        # leave room for activations / workspaces
        budget = free * self.ecfg.kv_fraction - 4 * (1 << 30)
        need = self.ecfg.max_running * ((self.ecfg.max_model_len + self.ecfg.page_size - 1)
                                        // self.ecfg.page_size)
        return int(max(64, min(budget // per_page, need)))

    # ------------------------------------------------------------------ API
    def export_prefix(self, tokens):
        """PrefixSnapshot of the cached KV pages of `tokens` (engine/prefix_share.py)."""
        from .prefix_share import export_prefix
        return export_prefix(self, tokens)

    def import_prefix(self, snapshot) -> int:
        """Load a PrefixSnapshot into this engine's prefix cache; returns the
        number of tokens newly cached."""
        from .prefix_share import import_prefix
        return import_prefix(self, snapshot)

    def recent_prompts(self) -> list:
        """Prompts of recently released requests, newest last (the candidates
        for persisting the prefix cache)."""
        return [p.tolist() for p in self._recent.values()]

    def save_prefix_cache(self, path: str) -> int:
        """Persist the cached prefixes of recent prompts (build-stamped file)."""
        from .prefix_share import save_prefix_cache
        return save_prefix_cache(self, path)

    def load_prefix_cache(self, path: str) -> int:
        """Load a file of save_prefix_cache; a file of another build is discarded."""
        from .prefix_share import load_prefix_cache
        return load_prefix_cache(self, path)

    def load_lora(self, adapter, name: str | None = None) -> str:
        """Register a LoRA adapter (a LoraAdapter or a LoRA GGUF path) for
        requests to select by name."""
        from ..models.lora import LoraAdapter
        if isinstance(adapter, str):
            adapter = LoraAdapter.from_gguf(adapter, name)
        if name:
            adapter.name = name
        if adapter.name in self.lora_names:
            return adapter.name
        if getattr(self.model, "lora", None) is not None:
            slot = self.model.lora.add(adapter)
        elif hasattr(self.model, "lora_adapters"):
            ads = self.model.lora_adapters
            slot = ads.index(None) if None in ads else len(ads)
            if slot == len(ads):
                ads.append(adapter)
            else:
                ads[slot] = adapter
        else:
            raise RuntimeError("engine built without LoRA slots (EngineConfig.max_loras)")
        # a request's adapter id is its slot: the name list mirrors the slots
        while len(self.lora_names) <= slot:
            self.lora_names.append(None)
        self.lora_names[slot] = adapter.name
        return adapter.name

    def unload_lora(self, name: str) -> int:
        """Free an adapter's slot; refused while a live request uses it."""
        if name not in self.lora_names:
            raise KeyError(name)
        slot = self.lora_names.index(name)
        if slot in self.lora_of.values():
            raise RuntimeError(f"adapter {name!r} is in use by a running request")
        if getattr(self.model, "lora", None) is not None:
            self.model.lora.remove(name)
        else:
            self.model.lora_adapters[slot] = None
        self.lora_names[slot] = None
        return slot

    def adapters(self) -> list[str]:
        return [n for n in self.lora_names if n is not None]

    def load_vision(self, mmproj_path: str):
        """Image encoder for prompts with images (an mmproj GGUF)."""
        from ..models.vision import VisionEncoder
        self.vision = VisionEncoder.from_gguf(mmproj_path, self.cfg.hidden, device=self.device)
        return self.vision

    def _splice_images(self, prompt_ids, images):
        """Each IMAGE_TOKEN in the prompt becomes the image's rows: placeholder
        ids (derived from the rows, for the prefix cache) whose embeddings the
        runner replaces with the encoder's rows."""
        from ..models.vision import IMAGE_TOKEN, image_placeholders
        if self.vision is None:
            raise RuntimeError("no image encoder loaded (load_vision / --mmproj)")
        if sum(1 for t in prompt_ids if t == IMAGE_TOKEN) != len(images):
            raise ValueError("the prompt must carry one image marker per image")
        ids, spans, k = [], [], 0
        for t in prompt_ids:
            if t == IMAGE_TOKEN:
                rows = self.vision.encode([images[k]])
                k += 1
                spans.append((len(ids), rows.to(self.device)))
                ids.extend(image_placeholders(rows, rows.shape[0], self.cfg.vocab))
            else:
                ids.append(int(t))
        return ids, spans

    def add_request(self, prompt_ids, params: SamplingParams | None = None,
                    request_id: int | None = None, lora: str | None = None,
                    images=None) -> int:
        params = params or SamplingParams()
        rid = next(self._ids) if request_id is None else request_id
        if images:
            prompt_ids, spans = self._splice_images(list(prompt_ids), images)
            self.images[rid] = spans
        if lora is not None:
            self.lora_of[rid] = self.lora_names.index(lora)
        eos = -1 if params.ignore_eos else params.eos_token_id
        salt = cache_salt(lora)
        if self.state_cache is not None:
            self._add_hybrid(rid, prompt_ids, params, eos, salt)
        else:
            self.sched.add_request(rid, [int(t) for t in prompt_ids], int(params.max_tokens),
                                   int(eos), salt)
        if lora is None and self.ecfg.prefix_cache:
            self._prompts[rid] = np.asarray(prompt_ids, dtype=np.int32)
        self.params[rid] = params
        if params.penalized:
            self._gen_counts[rid] = collections.Counter()
        self.prompt_len[rid] = len(prompt_ids)
        self.traces[rid] = RequestTrace(rid, len(prompt_ids))
        return rid

    def _add_hybrid(self, rid, prompt_ids, params, eos, salt):
        """Admission of a hybrid-model request: a prefix hit only where a
        recurrent state was saved, and a chunk split where one will be."""
        ps = self.bm.page_size
        toks = [int(t) for t in prompt_ids]
        npg = (len(toks) - 1) // ps
        hashes = [int(h) for h in self.bm.chain_hashes(toks, npg, salt)] if npg > 0 else []
        i = self.state_cache.deepest(hashes)
        cover = (i + 1) * ps if i >= 0 else 0
        split = npg * ps if npg * ps > cover else -1
        self.sched.add_request(rid, toks, int(params.max_tokens), int(eos), salt, cover, True, split)
        self._hyb[rid] = {"restore": (cover, hashes[i]) if cover else None,
                          "save": (split, hashes[npg - 1]) if split > 0 else None}

    def _hybrid_before(self, plan):
        for b, sid in enumerate(plan.seq_ids):
            h = self._hyb.get(int(sid))
            if h is None or h["restore"] is None:
                continue
            cover, key = h["restore"]
            h["restore"] = None
            if int(plan.positions[int(plan.seq_start[b])]) == cover:  # the hit happened
                self.state_cache.restore(key, self.runner.slots.get(int(sid)))

    def _hybrid_after(self, plan):
        for b, sid in enumerate(plan.seq_ids):
            h = self._hyb.get(int(sid))
            if h is None or h["save"] is None:
                continue
            at, key = h["save"]
            r0, n = int(plan.seq_start[b]), int(plan.seq_ntok[b])
            if n and int(plan.positions[r0]) + n == at:
                h["save"] = None
                self.state_cache.save(key, self.runner.slots.get(int(sid)))

    def abort(self, rid: int):
        self._hyb.pop(rid, None)
        self._gen_counts.pop(rid, None)
        self.sched.abort(rid)
        self._free_state(rid)
        self.images.pop(rid, None)
        self._prompts.pop(rid, None)

    def _free_state(self, rid: int):
        slots = getattr(self.runner, "slots", None)
        if slots is not None:
            slots.release(rid)

    def has_work(self) -> bool:
        return self.sched.has_work()

    def step(self) -> list[tuple[int, int, bool]]:
        """One engine iteration.  Returns (request_id, new_token, finished) for
        every request that produced a token."""
        plan = self.sched.schedule()
        if len(plan) == 0:
            return []
        ids = [int(s) for s in plan.seq_ids]
        samp = plan.seq_sample
        params = [self.params[i] for i, s in zip(ids, samp) if s]
        history = ([self._gen_counts.get(i) for i, s in zip(ids, samp) if s]
                   if self._gen_counts else None)
        if self.state_cache is not None:
            self._hybrid_before(plan)
        with self.profiler.stage("forward"):
            sampled = self.runner.run(plan, self.bm, params, history)
        if self.state_cache is not None:
            self._hybrid_after(plan)
        if any(p.constraint is not None for p in params):
            sampled = self._constrain(params, sampled)
        done = set(int(d) for d in self.sched.commit(plan, sampled.tolist()))
        out = []
        now = time.perf_counter()
        k = 0
        for i, s in zip(ids, samp):
            if not s:
                continue
            tok = int(sampled[k])
            k += 1
            cnt = self._gen_counts.get(i)
            if cnt is not None:
                cnt[tok] += 1
            tr = self.traces.get(i)
            if tr is not None:
                tr.on_token(now)
            out.append((i, tok, i in done))
        self.steps += 1
        return out

    def _constrain(self, params, sampled):
        """Apply per-request token constraints to the sampled rows: keep the
        drawn token if allowed, else the best allowed candidate by logit (the
        top 64, then the whole row).  Runs before the scheduler commits."""
        from .sampling import constrained_token
        sampled = np.array(sampled, copy=True)
        logits = self.runner.last_logits
        for k, p in enumerate(params):
            if p.constraint is not None:
                sampled[k] = constrained_token(p.constraint, int(sampled[k]), logits[k],
                                               p.eos_token_id)
        return sampled

    def embed_text(self, ids: list[int]) -> list[float]:
        """Mean-pooled, L2-normalised input embeddings of a token list (the
        /v1/embeddings route)."""
        if not ids:
            return [0.0] * self.cfg.hidden
        m = self.model
        if self.device.type == "cuda":
            from ..utils.ext import C
            t = torch.tensor(ids, dtype=torch.int32, device=self.device)
            out = torch.empty(len(ids), self.cfg.hidden, dtype=torch.float32, device=self.device)
            C().embed_gather(m.embd, m.embd_type, self.cfg.hidden, t, out)
            v = out.mean(0)
        else:
            v = m.embd[torch.tensor(ids)].float().mean(0)
        v = v / (v.norm() + 1e-12)
        return v.cpu().tolist()

    def output(self, rid: int) -> list[int]:
        return [int(t) for t in self.sched.output(rid)]

    def release(self, rid: int):
        self.sched.release(rid)
        self._free_state(rid)
        self.lora_of.pop(rid, None)
        self.images.pop(rid, None)
        self.params.pop(rid, None)
        self.prompt_len.pop(rid, None)
        self._hyb.pop(rid, None)
        self._gen_counts.pop(rid, None)
        p = self._prompts.pop(rid, None)
        if p is not None and len(p) >= self.bm.page_size:
            key = p.tobytes()
            self._recent.pop(key, None)
            self._recent[key] = p
            while len(self._recent) > RECENT_PROMPTS:
                self._recent.popitem(last=False)

    def generate(self, prompts: list[list[int]], params: SamplingParams | list[SamplingParams] | None = None
                 ) -> list[RequestOutput]:
        if not isinstance(params, list):
            params = [params or SamplingParams()] * len(prompts)
        # a constraint carries per-request state: each request gets its own
        params = [dataclasses.replace(sp, constraint=sp.constraint.fresh())
                  if sp.constraint is not None else sp for sp in params]
        rids = [self.add_request(p, sp) for p, sp in zip(prompts, params)]
        pending = set(rids)
        results: dict[int, list[int]] = {r: [] for r in rids}
        while pending:
            for rid, tok, fin in self.step():
                if rid in results:
                    results[rid].append(tok)
                if fin:
                    pending.discard(rid)
            if not self.sched.has_work() and pending:
                raise RuntimeError("scheduler idle with pending requests")
        outs = []
        for r in rids:
            tr = self.traces.pop(r, None)
            if tr:
                tr.finish(time.perf_counter())
            outs.append(RequestOutput(r, self.prompt_len[r], results[r], True, tr))
            self.release(r)
        return outs
