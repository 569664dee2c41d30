"""Multi-GPU arm of bench.py: Llama-3.3-70B pipeline-split over N ranks
(torchrun, one process per GPU, NCCL p2p between stages).

Weak scaling: 32 sequences per stage in flight (global batch 32*N), cut into
N micro-batches.  Device time is CUDA events around exactly K engine steps
on every rank (barrier + synchronize on both sides), reduced with MAX.
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
        print(f"[bench-pp {time.strftime('%H:%M:%S')}] {msg}", file=sys.stderr, flush=True)


def pipeline_bench(args):
    from bench import BASELINE_70B_TOKS, ClockSampler
    from ..engine import EngineConfig, SamplingParams
    from ..models.config import preset
    from ..models.weights import RandomSource
    from .pipeline import PipelineEngine, init_distributed

    init_distributed("nccl", timeout_s=600)
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device(f"cuda:{int(os.environ.get('LOCAL_RANK', 0))}")
    cfg = preset(args.model)
    if args.layers:
        cfg = cfg.scaled(n_layers=args.layers)
    tp = getattr(args, "tp", 1) or 1
    n_stages = world // tp
    B = args.batch * n_stages
    P, G = args.prompt, args.gen
    ecfg = EngineConfig(max_model_len=P + G + 64, max_running=B, max_step_tokens=P,
                        prefill_chunk=P, kv_pages=B * ((P + G + 64 + 15) // 16) + 64)
    t0 = time.time()
    eng = PipelineEngine(cfg, ecfg, lambda: RandomSource(cfg, seed=1234, on_device=True), dev,
                         micro_batches=n_stages, tp=tp)
    torch.cuda.synchronize()
    dist.barrier()
    _log(rank, f"stages {eng.bounds}, init {time.time() - t0:.1f}s")
    rng = np.random.default_rng(0)
    sp = SamplingParams(max_tokens=G, ignore_eos=True)

    def run_until(cond):
        while True:
            flag = torch.tensor([1 if (rank != 0 or cond()) else 0], dtype=torch.int32, device=dev)
            dist.all_reduce(flag, op=dist.ReduceOp.MIN)
            if not flag.item():
                return
            eng.step()

    # ---- TTFT: one prompt alone, through the public API
    ttfts = []
    for r in range(args.ttft_reps + 1):
        torch.cuda.synchronize()
        dist.barrier()
        t = time.perf_counter()
        rid = eng.add_request(rng.integers(0, cfg.vocab, P).tolist(),
                              SamplingParams(max_tokens=1, ignore_eos=True)) if rank == 0 else None
        run_until(lambda: len(eng.output(rid)) == 0)
        ttfts.append((time.perf_counter() - t) * 1e3)
        if rank == 0:
            eng.sched.release(rid)
    _log(rank, f"ttft (ms) {[round(x, 1) for x in ttfts]}")

    def decode(batch):
        rids = []
        if rank == 0:
            rids = [eng.add_request(rng.integers(0, cfg.vocab, P).tolist(), sp) for _ in range(batch)]
        t_pf = time.time()
        run_until(lambda: eng.sched.num_waiting > 0 or any(len(eng.output(x)) == 0 for x in rids))
        _log(rank, f"batch {batch}: prefill {time.time() - t_pf:.1f}s")
        for _ in range(args.warmup):
            eng.step()
        torch.cuda.synchronize()
        dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(0) as cs:
            t = time.perf_counter()
            a.record()
            for _ in range(args.steps):
                eng.step()
            b.record()
            torch.cuda.synchronize()
            wall = time.perf_counter() - t
        dist.barrier()
        ms = torch.tensor([a.elapsed_time(b)], device=dev)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        wl = torch.tensor([wall], device=dev)
        dist.all_reduce(wl, op=dist.ReduceOp.MAX)
        if rank == 0:
            for x in rids:
                eng.sched.abort(x)
                eng.sched.release(x)
        return float(ms.item()), float(wl.item()), cs.summary()

    ms_b, wall_b, clocks = decode(B)
    ms_1, wall_1, _ = decode(1)
    value = B * args.steps / (ms_b / 1e3)
    # every rank runs its stage's forward once per micro-batch
    launches = torch.tensor([eng.model.decode_launches() * eng.micro * args.steps], device=dev)
    dist.all_reduce(launches)
    if rank == 0:
        line = {
            "metric": f"decode tok/s at batch {args.batch} per stage (aggregate), Llama-3.3-70B Q4_K",
            "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_b / args.steps, 4),
            "higher_is_better": True, "scaling": "weak",
            "vs_baseline": round(value / BASELINE_70B_TOKS, 2),
            "dtype": "fp16 activations, fp32 accumulate, Q4_K weights",
            "data": "synthetic uniform-random token ids; random-init Q4_K weights (llama-3.3-70b architecture)",
            "config": {"model": cfg.name, "layers": cfg.n_layers, "global_batch": B, "seq_len": P,
                       "gen_len": G,
                       "parallelism": f"pp{n_stages}" + (f"xtp{tp}" if tp > 1 else ""),
                       "stages": eng.bounds, "micro_batches": eng.micro,
                       "tp": "fused: GEMM epilogue pushes partials over NVLink" if tp > 1 else None,
                       "kv": "paged fp16, 16-token pages",
                       "l2": "no flush: weights streamed per step >> 126 MB L2"},
            "decode_tok_s_batch1": round(args.steps / (ms_1 / 1e3), 2),
            "ttft_p50_ms": round(statistics.median(ttfts[1:]), 2), "ttft_prompt_tokens": P,
            "e2e": {"value": round(B * args.steps / wall_b, 2), "unit": "tokens/s",
                    "h2d_bytes_per_step": int(4 * (4 + eng.max_pages) * B + 12),
                    "d2h_bytes_per_step": 4 * B},
            "gpu_launches": int(launches.item()),
            "clocks": clocks,
        }
        if args.layers:
            line["invalid"] = "layer count overridden (debug)"
        print(json.dumps(line), flush=True)
    dist.barrier()
    dist.destroy_process_group()
