"""The split check: the tiny Llama (2 layers, Q4_0) run once in one process
and once split layer by layer over `world` local CPU processes (gloo);
greedy tokens must be equal and logits equal to within 1e-5.  Backs the CLI
`test-split` and the CPU pipeline test.

Reference behaviour: `swarmllm test-split` (src/main.rs:171; CPU split across
local daemons).
"""
from __future__ import annotations

import os
import socket
import tempfile

import numpy as np


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out_dir, micro, n_prompts, prompt_len, gen, native=False):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    import torch
    import torch.distributed as dist
    torch.set_num_threads(2)
    from ..engine import EngineConfig, SamplingParams
    from ..models.config import tiny_llama
    from ..models.weights import RandomSource
    from .pipeline import PipelineEngine, init_distributed
    init_distributed("gloo", timeout_s=120)
    cfg = tiny_llama()
    ecfg = EngineConfig(max_model_len=128, max_running=4, max_step_tokens=256, prefill_chunk=64,
                        cpu_native=native)
    eng = PipelineEngine(cfg, ecfg, lambda: RandomSource(cfg, seed=42), "cpu", micro_batches=micro)
    if eng.last:
        eng.record_logits = []
    rng = np.random.default_rng(7)
    prompts = [rng.integers(0, cfg.vocab, prompt_len).tolist() for _ in range(n_prompts)]
    toks = eng.generate(prompts, SamplingParams(max_tokens=gen))
    if eng.last:
        torch.save(eng.record_logits, os.path.join(out_dir, f"logits_w{world}.pt"))
    if eng.first:
        torch.save(toks, os.path.join(out_dir, f"tokens_w{world}.pt"))
        torch.save((eng.segments_served, eng.bytes_sent), os.path.join(out_dir, f"stats_w{world}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def split_check(world: int = 2, micro: int = 2, n_prompts: int = 4, prompt_len: int = 32,
                gen: int = 64, native: bool = False) -> dict:
    """`native`: both runs on the native CPU kernels (Q4_0 weights through the
    int8 matmul, native attention) instead of the fp32 PyTorch path."""
    import torch
    import torch.multiprocessing as mp
    with tempfile.TemporaryDirectory() as d:
        for w in (1, world):
            mp.start_processes(_worker, args=(w, _free_port(), d, micro, n_prompts, prompt_len, gen,
                                              native),
                               nprocs=w, join=True, start_method="spawn")
        t1, t2 = (torch.load(os.path.join(d, f"tokens_w{w}.pt")) for w in (1, world))
        l1, l2 = (torch.load(os.path.join(d, f"logits_w{w}.pt")) for w in (1, world))
        segs, sent = torch.load(os.path.join(d, f"stats_w{world}.pt"))
    worst = max((float((a - b).abs().max()) for a, b in zip(l1, l2)), default=float("inf"))
    ok = t1 == t2 and len(l1) == len(l2) and worst <= 1e-5
    return {"world": world, "native": native, "tokens_equal": t1 == t2, "steps": len(l1),
            "first_stage_segments": segs, "first_stage_bytes_sent": sent,
            "max_logit_diff": worst, "tokens": t1, "ok": ok}
