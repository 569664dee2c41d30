"""Multi-GPU arm of bench.py for dense models: Llama-3.3-70B pipeline-split
over N / tp stages (torchrun, one process per GPU, NCCL p2p between stages),
tensor-parallel inside each stage when tp > 1, run by the wave-pipelined
engine (parallel/async_pipeline.py).

Strong scaling: the global batch is `batch` sequences (32) at every N, split
into min(stages, batch) waves; the batch-1 figure is one sequence alone, and
the TTFT one prompt alone.  Device time: CUDA events on every rank around
exactly K decode steps of every running sequence (K wave steps per non-empty
wave) with barrier + synchronize on both sides, reduced with MAX; the same
steps run through the public API (requests in, sampled tokens out), so the
host wall time (MAX over ranks) is the end-to-end figure.
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


def _max(v: float, dev) -> float:
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def pipeline_bench(args):
    from bench import BASELINE_70B_TOKS, ClockSampler
    from ..engine import EngineConfig, SamplingParams
    from ..models.config import preset
    from ..models.weights import RandomSource
    from .async_pipeline import AsyncPipelineEngine
    from .pipeline import init_distributed

    init_distributed("nccl", timeout_s=600)
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device(f"cuda:{int(os.environ.get('LOCAL_RANK', 0))}")
    cfg = preset(args.model)
    if args.layers:
        cfg = cfg.scaled(n_layers=args.layers)
    tp = getattr(args, "tp", 1) or 1
    S = world // tp
    B = args.batch                      # global batch (all waves together)
    P, G = args.prompt, args.gen
    ecfg = EngineConfig(max_model_len=P + G + 64, max_running=B, max_step_tokens=P,
                        prefill_chunk=P, kv_pages=B * ((P + G + 64 + 15) // 16) + 64 * S)
    t0 = time.time()
    eng = AsyncPipelineEngine(cfg, ecfg, lambda: RandomSource(cfg, seed=1234, on_device=True),
                              dev, tp=tp, waves=min(S, B))
    torch.cuda.synchronize()
    dist.barrier()
    _log(rank, f"stages {eng.bounds} x tp{tp}, waves {eng.V}, init {time.time() - t0:.1f}s")
    rng = np.random.default_rng(0)
    sp = SamplingParams(max_tokens=G, ignore_eos=True)

    # ---- TTFT: one prompt alone through the public API
    ttfts = []
    for _ in range(args.ttft_reps + 1):
        torch.cuda.synchronize()
        dist.barrier()
        t = time.perf_counter()
        if rank == 0:
            rid = eng.add_request(rng.integers(0, cfg.vocab, P).tolist(),
                                  SamplingParams(max_tokens=1, ignore_eos=True))
            eng.run(stop_when=lambda: len(eng.output(rid)) > 0)
            eng.release(rid)
        else:
            eng.run()
        torch.cuda.synchronize()
        ttfts.append(_max((time.perf_counter() - t) * 1e3, dev))
    _log(rank, f"ttft (ms) {[round(x, 1) for x in ttfts]}")

    def decode(batch):
        rids = []
        if rank == 0:
            rids = [eng.add_request(rng.integers(0, cfg.vocab, P).tolist(), sp)
                    for _ in range(batch)]
        live = min(batch, eng.V)            # waves holding sequences
        t_pf = time.time()
        eng.run(stop_when=(lambda: all(len(eng.output(x)) > 0 for x in rids)) if rank == 0 else None)
        _log(rank, f"batch {batch}: prefill {time.time() - t_pf:.1f}s")
        if rank == 0:
            target = eng.retired + args.warmup * live
            eng.run(stop_when=lambda: eng.retired >= target)
        else:
            eng.run()
        torch.cuda.synchronize()
        dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(int(os.environ.get("LOCAL_RANK", 0))) as cs:
            t = time.perf_counter()
            a.record()
            if rank == 0:
                target = eng.retired + args.steps * live
                eng.run(stop_when=lambda: eng.retired >= target)
            else:
                eng.run()
            b.record()
            torch.cuda.synchronize()
            wall = time.perf_counter() - t
        ms = _max(a.elapsed_time(b), dev)
        wall = _max(wall, dev)
        if rank == 0:
            for x in rids:
                eng.abort(x)
                eng.release(x)
            eng.run()  # retire the aborted sequences (no work left: returns at once)
        else:
            eng.run()
        return ms, wall, cs.summary()

    ms_b, wall_b, clocks = decode(B)
    ms_1, wall_1, _ = decode(1)
    tokens = args.steps * B
    value = tokens / (ms_b / 1e3)
    launches = torch.tensor([eng.model.decode_launches() * args.steps * min(B, eng.V)], device=dev)
    dist.all_reduce(launches)
    if rank == 0:
        line = {
            "metric": f"decode tok/s at batch {B} (aggregate), Llama-3.3-70B Q4_K",
            "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_b / args.steps, 4),
            "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None,
            "vs_baseline_batch1": round(args.steps / (ms_1 / 1e3) / BASELINE_70B_TOKS, 2),
            "dtype": "fp16 activations, fp32 accumulate, Q4_K weights",
            "data": "synthetic uniform-random token ids; random-init Q4_K weights (llama-3.3-70b architecture)",
            "config": {"model": cfg.name, "layers": cfg.n_layers, "global_batch": B,
                       "seq_len": P, "gen_len": G,
                       "parallelism": f"pp{S}" + (f"xtp{tp}" if tp > 1 else ""),
                       "stages": eng.bounds, "waves": eng.V,
                       "step": "every running sequence advances one token",
                       "tp": "fused: GEMM epilogue pushes partials over NVLink" if tp > 1 else None,
                       "kv": "paged fp16, 16-token pages",
                       "l2": "no flush: weights streamed per step >> 126 MB L2"},
            "decode_tok_s_batch1": round(args.steps / (ms_1 / 1e3), 2),
            "ms_per_step_batch1": round(ms_1 / args.steps, 4),
            "ttft_p50_ms": round(statistics.median(ttfts[1:]), 2), "ttft_prompt_tokens": P,
            "e2e": {"value": round(tokens / wall_b, 2), "unit": "tokens/s",
                    "h2d_bytes_per_step": int(4 * (4 + eng.max_pages + 3) * B + 32 * min(B, eng.V)),
                    "d2h_bytes_per_step": 4 * B, "batch1_value": round(args.steps / wall_1, 2)},
            "gpu_launches": int(launches.item()),
            "clocks": clocks,
        }
        if args.layers:
            line["invalid"] = "layer count overridden (debug)"
        print(json.dumps(line), flush=True)
    dist.barrier()
    if eng.tpg is not None:
        eng.tpg.close()
    dist.destroy_process_group()
