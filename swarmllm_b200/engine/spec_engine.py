"""Speculative serving: LLMEngine's public API (add_request / step / output /
release / abort / generate) on top of speculative rounds, so the HTTP server,
the CLI and the benchmarks can serve a model with a drafter.

    ecfg = EngineConfig(draft_model="llama-3.2-1b", spec_depth=4, spec_width=4)
    eng = create_engine(preset("llama-3.3-70b"), "cuda:0", ecfg)

Each ``step()`` admits waiting requests (prefill of target and drafter; the
first token is sampled from the prefill), then runs one speculative round for
every running request: a draft tree of `spec_depth` levels x `spec_width`
children from the drafter model (engine/spec.py) -- a drafter preset or GGUF,
the target itself ("self"), or the target with a block of middle layers
skipped ("swift[:ratio]", engine/swift.py) -- or an n-gram chain looked up
in the request's own text when ``draft_model == "ngram"`` (engine/ngram_spec.py),
verified by one target forward.  A step reports every token it committed, so
a request can advance several tokens per step.  Greedy and sampled requests
(temperature / top-k / top-p, Philox-coupled noise) are both served; their
output is what the non-speculative engine would produce.

Not served here (the plain LLMEngine serves them): LoRA adapters, images,
logit bias / penalties, JSON constraints, prefix caching.

Reference behaviour: the reference runs speculative decoding inside its
pipeline executor and model worker (draft trees, DSD, n-gram lookup:
src/inference/pipeline/dsd_tree.rs, src/inference/model_worker.rs:4131,
src/inference/draft_tree.rs:92); its DSD controller picks the draft length
from measured costs (src/inference/dsd_controller.rs:22), which SpecController
mirrors for the tree depth.
"""
from __future__ import annotations

import collections
import dataclasses
import itertools
import time

import torch

from ..models.config import ModelConfig, preset
from ..utils.tracing import RequestTrace
from .sampling import SamplingParams


class SpecController:
    """Picks the draft depth from measured acceptance and costs.

    A round of depth D costs about t_draft * D + t_verify and commits
    E[D] = sum_{i=0..D} a^i tokens for a per-level acceptance rate a (the
    expected accepted prefix of a chain plus the bonus token).  The depth
    with the most tokens per second wins; acceptance is an exponential
    moving average over rounds, so the depth follows the text being written.
    Reference: the DSD controller sizes its guess count from measured draft
    and verify costs (src/inference/dsd_controller.rs:22,91).
    """

    def __init__(self, max_depth: int, alpha: float = 0.2):
        self.max_depth = max_depth
        self.alpha = alpha
        self.accept = 0.6        # prior per-level acceptance
        self.t_draft = None      # seconds per drafter level
        self.t_verify = None     # seconds per target verify

    def observe(self, depth: int, accepted: int, t_draft: float, t_verify: float):
        if depth <= 0:
            return
        # a chain of depth D accepting k levels: estimate a from k / D, bounded
        rate = min(0.98, max(0.02, accepted / depth))
        self.accept = (1 - self.alpha) * self.accept + self.alpha * rate
        td = t_draft / depth
        self.t_draft = td if self.t_draft is None else (1 - self.alpha) * self.t_draft + self.alpha * td
        self.t_verify = (t_verify if self.t_verify is None
                         else (1 - self.alpha) * self.t_verify + self.alpha * t_verify)

    def expected_tokens(self, depth: int) -> float:
        a = self.accept
        return sum(a ** i for i in range(depth + 1))

    def best_depth(self) -> int:
        if self.t_draft is None:
            return self.max_depth
        best, best_rate = 1, 0.0
        for d in range(1, self.max_depth + 1):
            rate = self.expected_tokens(d) / (self.t_draft * d + self.t_verify)
            if rate > best_rate:
                best, best_rate = d, rate
        return best

    def break_even_accept(self, depth: int) -> float:
        """Per-level acceptance at which a depth-`depth` round commits as many
        tokens per second as plain decoding (one token per t_verify)."""
        if self.t_draft is None:
            return float("nan")
        cost = (self.t_draft * depth + self.t_verify) / self.t_verify
        lo, hi = 0.0, 1.0
        for _ in range(50):
            mid = (lo + hi) / 2
            if sum(mid ** i for i in range(depth + 1)) < cost:
                lo = mid
            else:
                hi = mid
        return hi


class SpecEngine:
    def __init__(self, decoder, cfg: ModelConfig, ecfg, adaptive: bool = True):
        self.dec = decoder
        self.cfg, self.ecfg = cfg, ecfg
        self.max_running = ecfg.max_running
        self.waiting: collections.deque = collections.deque()
        self.running: dict[int, object] = {}    # request id -> decoder sequence
        self.finished: dict[int, object] = {}
        self.params: dict[int, SamplingParams] = {}
        self.traces: dict[int, RequestTrace] = {}
        self.prompt_len: dict[int, int] = {}
        self._reported: dict[int, int] = {}
        self._ids = itertools.count()
        self.steps = 0
        depth = getattr(decoder, "depth", 1)
        self.controller = SpecController(depth) if adaptive and hasattr(decoder, "width") else None

    # ------------------------------------------------------------------ construction
    @classmethod
    def from_config(cls, cfg: ModelConfig, device="cuda:0", ecfg=None, source=None, seed: int = 0,
                    drafter_source=None):
        from ..models.llama import LlamaGPU
        from ..models.weights import RandomSource
        from .engine import EngineConfig
        from .ngram_spec import NgramSpecDecoder
        from .spec import TreeSpecDecoder
        ecfg = ecfg or EngineConfig()
        dev = torch.device(device)
        if dev.type != "cuda":
            raise ValueError("speculative serving runs on a GPU")
        target = LlamaGPU(cfg, source or RandomSource(cfg, seed=seed, on_device=True), dev)
        if ecfg.draft_model == "ngram":
            dec = NgramSpecDecoder(target, depth=ecfg.spec_depth, max_seqs=ecfg.max_running,
                                   max_model_len=ecfg.max_model_len,
                                   prefill_chunk=ecfg.prefill_chunk)
        else:
            if ecfg.draft_model == "self":      # the target drafts for itself: acceptance bound
                drafter = target
            elif ecfg.draft_model.startswith("swift"):  # "swift" or "swift:<skip ratio>"
                from .swift import layer_skip_drafter, skip_patterns
                ratio = float(ecfg.draft_model.split(":", 1)[1]) if ":" in ecfg.draft_model else 0.45
                drafter = layer_skip_drafter(target, skip_patterns(len(target.layers), ratio)[0])
            elif ecfg.draft_model.endswith(".gguf") or "/" in ecfg.draft_model:
                from ..models.weights import GgufSource
                dsrc = GgufSource(ecfg.draft_model)
                drafter = LlamaGPU(dsrc.cfg, dsrc, dev)
            else:
                dcfg = preset(ecfg.draft_model).scaled(vocab=cfg.vocab)
                drafter = LlamaGPU(dcfg, drafter_source or RandomSource(dcfg, seed=seed + 1,
                                                                        on_device=True), dev)
            dec = TreeSpecDecoder(target, drafter, depth=ecfg.spec_depth, width=ecfg.spec_width,
                                  max_seqs=ecfg.max_running, max_model_len=ecfg.max_model_len,
                                  prefill_chunk=ecfg.prefill_chunk)
        eng = cls(dec, cfg, ecfg)
        eng.model = target
        return eng

    # ------------------------------------------------------------------ API
    def add_request(self, prompt_ids, params: SamplingParams | None = None,
                    request_id: int | None = None, lora: str | None = None, images=None) -> int:
        if lora is not None or images:
            raise ValueError("the speculative engine serves base-model text requests")
        params = params or SamplingParams()
        if params.penalized:
            raise ValueError("penalties and logit bias are not served speculatively")
        if params.constraint is not None and not getattr(self.dec, "constrained", False):
            raise ValueError("constrained replies are served by the draft-tree speculator only")
        rid = next(self._ids) if request_id is None else request_id
        self.waiting.append((rid, [int(t) for t in prompt_ids]))
        self.params[rid] = params
        self.prompt_len[rid] = len(prompt_ids)
        self.traces[rid] = RequestTrace(rid, len(prompt_ids))
        return rid

    def has_work(self) -> bool:
        return bool(self.waiting) or any(not s.done for s in self.running.values())

    def output(self, rid: int) -> list[int]:
        s = self.running.get(rid) or self.finished.get(rid)
        return list(s.out) if s is not None else []

    def _drop(self, rid: int):
        s = self.running.pop(rid, None)
        if s is not None:
            self.dec.free(s)
            self.finished[rid] = s

    def abort(self, rid: int):
        self.waiting = collections.deque((r, p) for r, p in self.waiting if r != rid)
        self._drop(rid)

    def release(self, rid: int):
        self.abort(rid)
        self.finished.pop(rid, None)
        self.params.pop(rid, None)
        self.prompt_len.pop(rid, None)
        self._reported.pop(rid, None)

    def step(self) -> list[tuple[int, int, bool]]:
        """Admit waiting requests, run one speculative round; returns
        (request id, token, finished) for every committed token."""
        now0 = time.perf_counter()
        while self.waiting and len(self.running) < self.max_running:
            rid, prompt = self.waiting.popleft()
            p = self.params[rid]
            self.running[rid] = self.dec.add(prompt, int(p.max_tokens), p)
            self._reported[rid] = 0
        live = [s for s in self.running.values() if not s.done]
        if live:
            if self.controller is not None:
                self.dec.depth = self.controller.best_depth()
                self.dec.n_nodes = 1 + self.dec.depth * self.dec.width
            st = self.dec.stats
            r0, a0, s0 = st.rounds, st.accepted, st.seconds
            self.dec.step(live)
            if self.controller is not None and st.rounds > r0:
                per = max(1, len(live))
                dt = st.seconds - s0
                td = getattr(self.dec, "last_draft_s", dt * 0.3)
                self.controller.observe(self.dec.depth, (st.accepted - a0) / per, td, dt - td)
        out = []
        now = time.perf_counter()
        for rid, s in list(self.running.items()):
            k = self._reported[rid]
            new = s.out[k:]
            self._reported[rid] = len(s.out)
            tr = self.traces.get(rid)
            for j, tok in enumerate(new):
                if tr is not None:
                    tr.on_token(now)
                out.append((rid, int(tok), s.done and j == len(new) - 1))
            if s.done:
                self._drop(rid)
        self.steps += 1
        self.last_step_s = time.perf_counter() - now0
        return out

    def generate(self, prompts, params=None):
        from .engine import RequestOutput
        if not isinstance(params, list):
            params = [params or SamplingParams()] * len(prompts)
        # one constraint per request, from its start
        params = [dataclasses.replace(sp, constraint=sp.constraint.fresh())
                  if sp is not None and sp.constraint is not None else sp for sp in params]
        rids = [self.add_request(p, sp) for p, sp in zip(prompts, params)]
        res = {r: [] for r in rids}
        pending = set(rids)
        while pending:
            for rid, tok, fin in self.step():
                if rid in res:
                    res[rid].append(tok)
                if fin:
                    pending.discard(rid)
        outs = []
        for r in rids:
            tr = self.traces.pop(r, None)
            if tr:
                tr.finish(time.perf_counter())
            outs.append(RequestOutput(r, self.prompt_len[r], res[r], True, tr))
            self.release(r)
        return outs


def create_engine(cfg: ModelConfig, device="cuda:0", ecfg=None, source=None, seed: int = 0, **kw):
    """The engine an EngineConfig asks for: speculative when it names a
    drafter (a preset name, "self" or "ngram"), the plain LLMEngine otherwise."""
    from .engine import EngineConfig, LLMEngine
    ecfg = ecfg or EngineConfig()
    if ecfg.draft_model:
        return SpecEngine.from_config(cfg, device, ecfg, source=source, seed=seed)
    return LLMEngine.from_config(cfg, device, ecfg, source=source, seed=seed, **kw)
