"""Multi-GPU arm of bench.py for MoE models: expert parallelism over N ranks
(torchrun, one process per GPU).  Attention is data parallel (each rank
serves its own batch), the experts of every MoE layer are split over the
ranks and exchanged through peer memory inside each layer.

Weak scaling: `batch` sequences per rank.  Device time: CUDA events around
exactly K decode-step graph replays on every rank (barrier + synchronize on
both sides), reduced with MAX; end to end: K engine steps through the public
API (pinned H2D inputs, D2H sampled tokens), host-timed, MAX over ranks.
"""
from __future__ import annotations

import json
import os
import statistics
import sys
import time

import numpy as np
import torch
import torch.distributed as dist


def _log(rank, msg):
    if rank == 0:
        print(f"[bench-ep {time.strftime('%H:%M:%S')}] {msg}", file=sys.stderr, flush=True)


def _max(v: float, dev) -> float:
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def ep_bench(args):
    from bench import ClockSampler
    from ..engine import EngineConfig, LLMEngine, SamplingParams
    from ..models.config import preset
    from .ep import EpGroup
    from .pipeline import init_distributed

    init_distributed("nccl", timeout_s=600)
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device(f"cuda:{int(os.environ.get('LOCAL_RANK', 0))}")
    torch.cuda.set_device(dev)
    cfg = preset(args.model)
    if args.layers:
        cfg = cfg.scaled(n_layers=args.layers)
    B, P, G = args.batch, args.prompt, args.gen
    chunk = args.chunk or P
    ecfg = EngineConfig(max_model_len=P + G + 64, max_running=B, max_step_tokens=chunk,
                        prefill_chunk=chunk, graph_sizes=(1, B))
    t0 = time.time()
    ep = EpGroup(rank, world, dev)
    eng = LLMEngine.from_config(cfg, dev, ecfg, seed=1234, ep=ep)
    torch.cuda.synchronize()
    dist.barrier()
    _log(rank, f"EP{world} engine ready in {time.time() - t0:.1f}s; local weights "
               f"{eng.model.weight_bytes() / 1e9:.1f} GB")
    rng = np.random.default_rng(1000 + rank)
    sp = SamplingParams(max_tokens=G, ignore_eos=True)

    ttfts = []
    for _ in range(args.ttft_reps + 1):
        torch.cuda.synchronize()
        dist.barrier()
        t = time.perf_counter()
        rid = eng.add_request(rng.integers(0, cfg.vocab, P).tolist(),
                              SamplingParams(max_tokens=1, ignore_eos=True))
        while not any(o[0] == rid for o in eng.step()):
            pass
        ttfts.append(_max((time.perf_counter() - t) * 1e3, dev))
        eng.release(rid)
    _log(rank, f"ttft (ms, max over ranks) {[round(x, 1) for x in ttfts]}")

    def decode(batch):
        rids = [eng.add_request(rng.integers(0, cfg.vocab, P).tolist(), sp) for _ in range(batch)]
        while eng.sched.num_waiting or any(len(eng.output(r)) == 0 for r in rids):
            eng.step()
        for _ in range(args.warmup):
            eng.step()
        g, _, _ = eng.runner.graphs[batch]
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        dist.barrier()
        with ClockSampler(rank) as cs:
            a.record()
            for _ in range(args.steps):
                g.replay()
            b.record()
            torch.cuda.synchronize()
            dev_ms = _max(a.elapsed_time(b), dev)
            dist.barrier()
            t = time.perf_counter()
            for _ in range(args.steps):
                eng.step()
            torch.cuda.synchronize()
            e2e_s = _max(time.perf_counter() - t, dev)
        for r in rids:
            eng.abort(r)
            eng.release(r)
        return dev_ms, e2e_s, cs.summary(), eng.runner.h2d_bytes, eng.runner.d2h_bytes

    ms_b, e2e_b, clocks, h2d, d2h = decode(B)
    ms_1, e2e_1, _, _, _ = decode(1)
    value = world * B * args.steps / (ms_b / 1e3)
    line = {
        "metric": f"decode tok/s at batch {B} per GPU (aggregate over {world} GPUs), {cfg.name}",
        "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_b / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": f"fp16/bf16 activations, fp32 accumulate, {cfg.expert_qtype or cfg.weight_qtype} experts",
        "data": f"synthetic uniform-random token ids; random-init weights ({cfg.name} architecture)",
        "config": {"model": cfg.name, "layers": cfg.n_layers, "global_batch": B * world,
                   "seq_len": P, "gen_len": G, "parallelism": f"ep{world} (attention dp{world})",
                   "l2": "no flush: expert weights streamed per step >> 126 MB L2"},
        "decode_tok_s_batch1_per_gpu": round(world * args.steps / (ms_1 / 1e3), 2),
        "ttft_p50_ms": round(statistics.median(ttfts[1:]), 2), "ttft_prompt_tokens": P,
        "e2e": {"value": round(world * B * args.steps / e2e_b, 2), "unit": "tokens/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": eng.model.decode_launches() * args.steps,
        "clocks": clocks,
    }
    if args.layers:
        line["invalid"] = "layer count overridden (debug)"
    if rank == 0:
        print(json.dumps(line), flush=True)
    eng.runner.graphs.clear()
    ep.close()
    dist.barrier()
    dist.destroy_process_group()
