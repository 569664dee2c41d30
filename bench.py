"""Headline benchmark: Llama-3.3-70B (Q4_K, random-init) decode tok/s at batch 32
and batch 1, plus p50 TTFT of a 2048-token prompt, on N B200s of one node.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...       (N > 1)

N = 1: the whole model on one GPU.  N > 1 (torchrun): the same global batch
of 32 sequences (strong scaling) on a tensor-parallel and/or pipeline layout
(``--tp`` ranks per stage, the rest pipeline stages over NCCL p2p; see
``swarmllm_b200.parallel.bench_pp``).  The batch-1 figure is one sequence
alone and the TTFT one 2048-token prompt alone, at every N.

`vs_baseline` is null: the reference publishes no batch-32 figure for this
model.  `vs_baseline_batch1` divides the batch-1 rate by the reference's
published 70B figure (4.1 tok/s, batch 1, three computers over a WAN), which
is on other hardware and only context.

`value` is device time: CUDA events around exactly K decode steps on the
launching stream, bracketed by barrier + synchronize, max over ranks.
`e2e` is the same metric through the public engine API (`LLMEngine.step` /
`PipelineEngine.step`), whose timed region includes the H2D copy of each
step's inputs from pinned memory and the D2H read of the sampled tokens.
Workload: synthetic uniform-random token ids, random-init weights of the
named architecture (no network for checkpoints).  The 40 GB of weights read
per step are far larger than L2 (126 MB), so no L2 flush is needed.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

BASELINE_70B_TOKS = 4.1  # reference's published 70B decode tok/s (README.md:186, WAN, 3 computers)


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--model", default="llama-3.3-70b")
    p.add_argument("--batch", type=int, default=32)
    p.add_argument("--prompt", type=int, default=2048)
    p.add_argument("--gen", type=int, default=512)
    p.add_argument("--ttft-reps", type=int, default=3)
    p.add_argument("--chunk", type=int, default=0, help="prefill chunk (0: whole prompt)")
    p.add_argument("--tp", type=int, default=0,
                   help="tensor-parallel ranks per pipeline stage (0: all GPUs in one TP group)")
    p.add_argument("--pp-layout", action="store_true",
                   help="run tp == N through the wave-pipelined engine (one stage) instead")
    p.add_argument("--spec", action="store_true",
                   help="tree speculative decoding bench (70B target + 1B drafter, one GPU)")
    p.add_argument("--advance", type=int, default=256,
                   help="untimed decode steps before timing (mid-generation context; >= warmup)")
    p.add_argument("--layers", type=int, default=0, help="debug only: override layer count (invalid for the headline)")
    return p.parse_args()


class ClockSampler:
    """nvidia-smi clocks + throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        ids = gpu_index if isinstance(gpu_index, (list, tuple)) else [gpu_index]
        self.idx = ",".join(str(i) for i in ids)
        self.samples = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.Q}",
                                      "--format=csv,noheader,nounits"], capture_output=True,
                                     text=True, timeout=5).stdout.strip()
                if out:
                    self.samples.append([x.strip() for x in out.split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        mhz = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for s in self.samples:
            for i, n in enumerate(names):
                if len(s) > 5 + i and s[5 + i].lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(mhz) if mhz else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(self.samples)}


def reference_arm(args):
    print(json.dumps({"impl": "reference", "unavailable":
                      "reference is a Rust/candle crate with no Python package; it cannot be "
                      "pip-installed into baseline/_ref and no cargo/rustc toolchain or crates "
                      "registry exists offline"}))


def log(msg):
    print(f"[bench {time.strftime('%H:%M:%S')}] {msg}", file=sys.stderr, flush=True)


def measure(eng, cfg, args, replay, gpu_ids, h2d_of, d2h_of):
    """TTFT, then batch-B and batch-1 decode, on an engine driven from this
    process (LLMEngine, or the root of a TpEngine).  `replay(batch, steps)`
    runs `steps` captured decode graphs of `batch` rows and returns this rank's
    device ms (CUDA events on the launching stream)."""
    import numpy as np
    import torch

    from swarmllm_b200.engine import SamplingParams
    B, P, G = args.batch, args.prompt, args.gen
    rng = np.random.default_rng(0)
    sp = SamplingParams(max_tokens=G, ignore_eos=True)

    # ---- p50 TTFT: one 2048-token prompt alone, through the public API
    ttfts = []
    for r in range(args.ttft_reps + 1):
        prompt = rng.integers(0, cfg.vocab, P).tolist()
        torch.cuda.synchronize()
        t = time.perf_counter()
        rid = eng.add_request(prompt, SamplingParams(max_tokens=1, ignore_eos=True))
        while True:
            outs = eng.step()
            if any(o[0] == rid for o in outs):
                break
        ttfts.append((time.perf_counter() - t) * 1e3)
        eng.release(rid)
    log(f"ttft runs (ms): {[round(t, 1) for t in ttfts]}")

    def decode_rate(batch: int, steps: int, warmup: int):
        rids = [eng.add_request(rng.integers(0, cfg.vocab, P).tolist(), sp) for _ in range(batch)]
        with ClockSampler(gpu_ids) as cs:
            # run until every sequence is decoding
            t_pf = time.time()
            while eng.sched.num_waiting or any(len(eng.output(r)) == 0 for r in rids):
                eng.step()
            log(f"batch {batch}: prefill of {batch}x{P} tokens took {time.time() - t_pf:.1f}s")
            # untimed steps: the W warm-up steps, then on to mid-generation context
            for _ in range(max(warmup, args.advance)):
                eng.step()
            ctx = P + len(eng.output(rids[0]))
            # device-timed: K graph replays of the decode step (inputs already resident)
            torch.cuda.synchronize()
            dev_ms = replay(batch, steps)
            # end to end through the public API (H2D inputs + D2H tokens every step)
            torch.cuda.synchronize()
            t = time.perf_counter()
            for _ in range(steps):
                eng.step()
            e2e_s = time.perf_counter() - t
        for r in rids:
            eng.abort(r)
            eng.release(r)
        return dev_ms, e2e_s, cs.summary(), h2d_of(), d2h_of(), ctx

    ms_b, e2e_b, clocks, h2d, d2h, ctx = decode_rate(B, args.steps, args.warmup)
    ms1, e2e1, _, _, _, _ = decode_rate(1, args.steps, args.warmup)
    return dict(ttfts=ttfts, ms_b=ms_b, e2e_b=e2e_b, clocks=clocks, h2d=h2d, d2h=d2h, ms1=ms1,
                e2e1=e2e1, ctx=ctx)


def result_line(cfg, args, m, n_gpus, parallelism, weight_gb, launches_per_step, extra=None):
    B, P, G = args.batch, args.prompt, args.gen
    value = B * args.steps / (m["ms_b"] / 1e3)
    headline = cfg.name == "llama-3.3-70b"
    wq = cfg.expert_qtype if cfg.n_experts else cfg.weight_qtype
    if cfg.quant_mix:
        wq = f"{wq} + Q6_K ({cfg.quant_mix} mix)"
    b1 = args.steps / (m["ms1"] / 1e3)
    line = {
        "metric": (f"decode tok/s at batch {B} (aggregate), Llama-3.3-70B Q4_K" if headline else
                   f"decode tok/s at batch {B} (aggregate), {cfg.name}"),
        "value": round(value, 2), "unit": "tokens/s", "n_gpus": n_gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(m["ms_b"] / args.steps, 4),
        "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None,
        "vs_baseline_batch1": round(b1 / BASELINE_70B_TOKS, 2) if headline else None,
        "dtype": f"fp16/bf16 activations, fp32 accumulate, {wq} weights",
        "data": f"synthetic uniform-random token ids; random-init {wq} weights ({cfg.name} architecture)",
        "config": {"model": cfg.name, "layers": cfg.n_layers, "global_batch": B, "seq_len": P,
                   "gen_len": G, "parallelism": parallelism, "kv": "paged fp16, 16-token pages",
                   "context_at_timing": m["ctx"],
                   "timing": "K replays of the captured decode step, CUDA events, max over ranks",
                   "l2": f"no flush: {weight_gb:.0f} GB of weights per step, streamed, >> 126 MB L2"},
        "decode_tok_s_batch1": round(b1, 2),
        "ms_per_step_batch1": round(m["ms1"] / args.steps, 4),
        "ttft_p50_ms": round(statistics.median(m["ttfts"][1:]), 2), "ttft_prompt_tokens": P,
        "e2e": {"value": round(B * args.steps / m["e2e_b"], 2), "unit": "tokens/s",
                "h2d_bytes_per_step": m["h2d"], "d2h_bytes_per_step": m["d2h"],
                "batch1_value": round(args.steps / m["e2e1"], 2)},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": m["clocks"],
    }
    if extra:
        line.update(extra)
    if args.layers:
        line["invalid"] = "layer count overridden (debug)"
    return line


def _visible_gpu(local: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    ids = [x for x in vis.split(",") if x.strip()]
    return int(ids[local]) if local < len(ids) and ids[local].strip().isdigit() else local


def _graph_replay(runner):
    import torch

    def replay(batch, steps):
        g = runner.graphs[batch][0]
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            g.replay()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b)
    return replay


def single_gpu(args):
    import torch

    from swarmllm_b200.engine import EngineConfig, LLMEngine
    from swarmllm_b200.models.config import preset

    cfg = preset(args.model)
    if args.layers:
        cfg = cfg.scaled(n_layers=args.layers)
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    B, P, G = args.batch, args.prompt, args.gen
    chunk = args.chunk or P
    ecfg = EngineConfig(max_model_len=P + G + 64, max_running=B, max_step_tokens=chunk,
                        prefill_chunk=chunk, graph_sizes=(1, B))
    t0 = time.time()
    eng = LLMEngine.from_config(cfg, dev, ecfg, seed=1234)
    t_init = time.time() - t0
    log(f"engine ready in {t_init:.1f}s; weights {eng.model.weight_bytes() / 1e9:.1f} GB, "
        f"kv pages {eng.bm.num_pages}")
    runner = eng.runner
    m = measure(eng, cfg, args, _graph_replay(runner), [_visible_gpu(0)],
                lambda: runner.h2d_bytes, lambda: runner.d2h_bytes)
    line = result_line(cfg, args, m, 1, "single GPU", eng.model.weight_bytes() / 1e9,
                       eng.model.decode_launches(), {"init_s": round(t_init, 1)})
    print(json.dumps(line), flush=True)


def tensor_parallel(args):
    """N GPUs, one tensor-parallel group: every rank holds 1/N of every layer."""
    import torch
    import torch.distributed as dist

    from swarmllm_b200.engine import EngineConfig
    from swarmllm_b200.models.config import preset
    from swarmllm_b200.models.weights import RandomSource
    from swarmllm_b200.parallel.pipeline import init_distributed
    from swarmllm_b200.parallel.tp_engine import TpEngine

    init_distributed("nccl", timeout_s=600)
    rank, world = dist.get_rank(), dist.get_world_size()
    cfg = preset(args.model)
    if args.layers:
        cfg = cfg.scaled(n_layers=args.layers)
    B, P, G = args.batch, args.prompt, args.gen
    chunk = args.chunk or P
    ecfg = EngineConfig(max_model_len=P + G + 64, max_running=B, max_step_tokens=chunk,
                        prefill_chunk=chunk, graph_sizes=(1, B))
    t0 = time.time()
    eng = TpEngine.create(cfg, ecfg, lambda: RandomSource(cfg, seed=1234, on_device=True))
    t_init = time.time() - t0
    local = int(os.environ.get("LOCAL_RANK", rank))
    replays = []
    if eng.root:
        log(f"tp{world} engine ready in {t_init:.1f}s; weights per rank "
            f"{eng.model.weight_bytes() / 1e9:.1f} GB, kv pages {eng.bm.num_pages}")

        def replay(batch, steps):
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            eng.replay(batch, steps, ev)
            torch.cuda.synchronize()
            ms = ev[0].elapsed_time(ev[1])
            replays.append(ms)
            return ms
        inner = eng.runner._inner
        m = measure(eng, cfg, args, replay, [_visible_gpu(i) for i in range(world)],
                    lambda: inner.h2d_bytes, lambda: inner.d2h_bytes)
        eng.stop()
    else:
        eng.follow(on_replay=replays.append)
    # device time: max over ranks of every timed replay
    t = torch.tensor(replays + [0.0] * (2 - len(replays)), dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=eng.cpu_group)
    if eng.root:
        m["ms_b"], m["ms1"] = float(t[0]), float(t[1])
        line = result_line(cfg, args, m, world, f"tp{world}",
                           eng.model.weight_bytes() * world / 1e9, eng.model.decode_launches() * world,
                           {"init_s": round(t_init, 1),
                            "tp": "row-parallel GEMM epilogue stores each tile into its owner's "
                                  "buffer over NVLink; fused reduce + residual + RMSNorm + "
                                  "residual all-gather kernel (P2P stores, epoch flags)"})
        print(json.dumps(line), flush=True)
    dist.barrier(group=eng.cpu_group)
    eng.close()
    dist.destroy_process_group()


def _json_only_stdout():
    """Keep stdout for the result line: libraries that write to file
    descriptor 1 from C (NCCL's version banner, for one) go to stderr, and
    Python's sys.stdout keeps a private handle on the real stdout."""
    sys.stdout.flush()
    real = os.fdopen(os.dup(1), "w", buffering=1)
    os.dup2(2, 1)
    sys.stdout = real


def main():
    _json_only_stdout()
    args = parse()
    if args.impl == "reference":
        return reference_arm(args)
    if args.spec:
        from swarmllm_b200.engine.bench_spec import spec_bench
        return spec_bench(args, log)
    if args.gpus == 1 and int(os.environ.get("WORLD_SIZE", "1")) == 1:
        return single_gpu(args)
    from swarmllm_b200.models.config import preset
    if preset(args.model).n_experts:
        from swarmllm_b200.parallel.bench_ep import ep_bench
        return ep_bench(args)
    world = int(os.environ.get("WORLD_SIZE", args.gpus))
    if not args.tp:  # default layout: one tensor-parallel group over all GPUs
        args.tp = world
    if args.tp == world and not args.pp_layout:
        return tensor_parallel(args)
    from swarmllm_b200.parallel.bench_pp import pipeline_bench
    return pipeline_bench(args)


if __name__ == "__main__":
    main()
