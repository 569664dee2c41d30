"""Tree speculative decoding on the headline model (`bench.py --spec`): the
Llama-3.3-70B-architecture target with a Llama-3.2-1B-architecture drafter,
draft trees of depth 4 x width 4 (17 nodes), random-init weights, one GPU.

Random-init weights make the drafter's guesses right only by chance, so a
tokens/s figure for it measures the cost of speculation, not its benefit.
The bench therefore reports the pieces that decide the speed-up on real
weights, at batch 1 and batch 32 (prompts of 2048 random ids):

* plain decode step time (one row per sequence) and the target's verify time
  for the 17 tree rows per sequence (same eager forward path), and their ratio;
* drafter time per tree level and per round;
* tokens per round and tokens/s with the random 1B drafter (chance acceptance)
  and with the target drafting for itself (every guess accepted: the upper
  bound of tokens per round);
* the break-even per-level acceptance rate: the rate at which a round commits
  as many tokens per second as plain decoding.

Device time: CUDA events around each phase, synchronised on both sides.
"""
from __future__ import annotations

import json
import time

import numpy as np
import torch


def _ev():
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def spec_bench(args, log):
    from ..models.config import preset
    from ..models.llama import LlamaGPU
    from ..models.weights import RandomSource
    from .spec import TreeSpecDecoder
    from .spec_engine import SpecController

    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    cfg = preset(args.model)
    if args.layers:
        cfg = cfg.scaled(n_layers=args.layers)
    dcfg = preset("llama-3.2-1b").scaled(vocab=cfg.vocab)
    depth, width = 4, 4
    P, steps = args.prompt, max(3, args.steps // 4)
    target = LlamaGPU(cfg, RandomSource(cfg, seed=1234, on_device=True), dev)
    drafter = LlamaGPU(dcfg, RandomSource(dcfg, seed=99, on_device=True), dev)
    rng = np.random.default_rng(0)
    results = {}
    for batch in (1, args.batch):
        for name, d in (("drafter_1b", drafter), ("self_draft", target)):
            spec = TreeSpecDecoder(target, d, depth=depth, width=width, max_seqs=batch,
                                   max_model_len=P + 256, prefill_chunk=min(P, 2048))
            seqs = [spec.add(rng.integers(0, cfg.vocab, P).tolist(), 10 ** 6) for _ in range(batch)]
            for _ in range(2):                     # warm-up rounds
                spec.step(seqs)
            st0 = (spec.stats.rounds, spec.stats.committed, spec.stats.accepted)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            draft_s = 0.0
            for _ in range(steps):
                spec.step(seqs)
                draft_s += spec.last_draft_s
            torch.cuda.synchronize()
            wall = time.perf_counter() - t0
            rounds = spec.stats.rounds - st0[0]
            committed = spec.stats.committed - st0[1]
            accepted = spec.stats.accepted - st0[2]
            # plain decode vs verify (17 rows per sequence), same eager forward
            side = spec.t
            # (rows re-write the KV of each sequence's last position: it is freed next)
            rows1, rows17 = [], []
            for s in seqs:
                slot = spec.t.phys(s.sid, [s.pos - 1])[0]
                rows1.append((s.sid, s.root, s.pos - 1, slot, s.pos, 0, 0))
                for _ in range(spec.n_nodes):
                    rows17.append((s.sid, s.root, s.pos - 1, slot, s.pos, s.pos - 1, 1))
            t_plain = t_verify = 0.0
            for rows, key in ((rows1, "plain"), (rows17, "verify")):
                side.forward(rows, list(range(len(rows))), tree=key == "verify")
                a, b = _ev()
                a.record()
                for _ in range(3):
                    side.forward(rows, list(range(len(rows))), tree=key == "verify")
                b.record()
                torch.cuda.synchronize()
                ms = a.elapsed_time(b) / 3
                if key == "plain":
                    t_plain = ms
                else:
                    t_verify = ms
            for s in seqs:
                spec.free(s)
            round_ms = wall * 1e3 / rounds
            draft_ms = draft_s * 1e3 / rounds
            ctl = SpecController(depth)
            ctl.observe(depth, 0, draft_ms / 1e3, t_verify / 1e3)
            r = {"round_ms": round(round_ms, 3), "draft_ms_per_round": round(draft_ms, 3),
                 "draft_ms_per_level": round(draft_ms / depth, 3),
                 "plain_step_ms": round(t_plain, 3), "verify_ms_17_rows": round(t_verify, 3),
                 "verify_over_plain": round(t_verify / t_plain, 3),
                 "tokens_per_round": round(committed / rounds / batch, 3),
                 "accepted_per_round": round(accepted / rounds / batch, 3),
                 "tok_s": round(committed / wall, 2),
                 "plain_tok_s": round(batch / (t_plain / 1e3), 2),
                 "break_even_accept_per_level": round(ctl.break_even_accept(depth), 3)}
            results[f"batch{batch}_{name}"] = r
            log(f"spec batch {batch} {name}: {r}")
            del spec
            torch.cuda.empty_cache()
    line = {"metric": "tree speculative decoding (depth 4 x width 4), Llama-3.3-70B Q4_K + "
                      "Llama-3.2-1B drafter", "unit": "see fields", "n_gpus": 1,
            "data": "synthetic random token ids; random-init weights (drafter acceptance is "
                    "chance: tokens/round with it measures the cost of speculating)",
            "config": {"model": cfg.name, "drafter": dcfg.name, "prompt": P, "depth": depth,
                       "width": width, "rounds_timed": steps,
                       "timing": "CUDA events; eager forwards (no graphs) on both sides"},
            "results": results}
    print(json.dumps(line), flush=True)
