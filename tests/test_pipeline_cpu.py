"""Two-CPU-peer split (plumbing, no GPU): the tiny Llama (2 layers, hidden 256,
4/2 heads, d 64, FFN 512, vocab 32000, Q4_0 weights, F32 norms) split layer 0 |
layer 1 across 2 local processes over gloo; 4 prompts of 32 random ids,
greedy decode of 64 tokens; logits must match a single-process run."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


@pytest.mark.timeout(600)
def test_two_peer_split_matches_single_peer():
    from swarmllm_b200.parallel.split_check import split_check
    r = split_check(world=2, micro=2)
    assert r["tokens_equal"], r
    assert all(len(t) == 64 for t in r["tokens"])
    assert r["max_logit_diff"] <= 1e-5, r["max_logit_diff"]
    assert r["ok"]
    # the first stage ran forwards and sent its activations on
    assert r["first_stage_segments"] > 0 and r["first_stage_bytes_sent"] > 0


@pytest.mark.timeout(600)
def test_two_peer_split_native_kernels():
    """The same split on the native CPU kernels (Q4_0 weights through the int8
    matmul, native attention): per-row arithmetic, so the split equals one
    process exactly."""
    from swarmllm_b200.parallel.split_check import split_check
    r = split_check(world=2, micro=2, gen=16, native=True)
    assert r["native"] and r["tokens_equal"] and r["max_logit_diff"] <= 1e-5, r


def test_stage_bounds():
    from swarmllm_b200.parallel.pipeline import stage_bounds
    b = stage_bounds(80, 8, 0.5, 1.0)
    assert b[0] == 0 and b[-1] == 80 and len(b) == 9
    sizes = [b[i + 1] - b[i] for i in range(8)]
    assert max(sizes) - min(sizes) <= 2
    assert stage_bounds(2, 2) == [0, 1, 2]


def _async_worker(rank, world, port, q, long_prompt=False):
    import os
    import torch
    import torch.distributed as dist
    torch.set_num_threads(1)
    from swarmllm_b200.engine.engine import EngineConfig
    from swarmllm_b200.engine.sampling import SamplingParams
    from swarmllm_b200.models.config import tiny_llama
    from swarmllm_b200.models.weights import RandomSource
    from swarmllm_b200.parallel.async_pipeline import AsyncPipelineEngine
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    cfg = tiny_llama().scaled(n_layers=3)
    ecfg = EngineConfig(max_model_len=128, max_running=6, max_step_tokens=64, prefill_chunk=16,
                        prefix_cache=False)
    eng = AsyncPipelineEngine(cfg, ecfg, lambda: RandomSource(cfg, seed=5), "cpu")
    rng = np.random.default_rng(4)
    lens = (60,) if long_prompt else (5, 30, 12, 21, 9)
    prompts = [rng.integers(0, cfg.vocab, n).tolist() for n in lens]
    out = eng.generate(prompts, SamplingParams(max_tokens=9, ignore_eos=True))
    if rank == 0:
        q.put((out, eng.chunks_pipelined) if long_prompt else out)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_async_waves_match_single_process(world):
    """Wave-pipelined split (independent waves, plan travelling with the
    activations, chunked prefill) == one process, token for token."""
    import multiprocessing as mp
    import socket
    from swarmllm_b200.engine import EngineConfig, LLMEngine, SamplingParams
    from swarmllm_b200.models.config import tiny_llama
    from swarmllm_b200.models.weights import RandomSource
    cfg = tiny_llama().scaled(n_layers=3)
    rng = np.random.default_rng(4)
    prompts = [rng.integers(0, cfg.vocab, n).tolist() for n in (5, 30, 12, 21, 9)]
    ref = LLMEngine.from_config(cfg, "cpu", EngineConfig(max_model_len=128, max_running=6,
                                                         max_step_tokens=64, prefill_chunk=16,
                                                         prefix_cache=False),
                                source=RandomSource(cfg, seed=5))
    want = [o.token_ids for o in ref.generate(prompts, SamplingParams(max_tokens=9,
                                                                      ignore_eos=True))]
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_async_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        got = q.get(timeout=240)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert got == want


def _async_long_worker(rank, world, port, q):
    _async_worker(rank, world, port, q, long_prompt=True)


def test_async_prompt_chunks_flow_through_stages():
    """One 60-token prompt in 16-token chunks over 3 stages: the chunks that
    sample nothing go down the chain one behind the other (not one at a time
    through every stage), and the output equals one process."""
    import multiprocessing as mp
    import socket
    from swarmllm_b200.engine import EngineConfig, LLMEngine, SamplingParams
    from swarmllm_b200.models.config import tiny_llama
    from swarmllm_b200.models.weights import RandomSource
    cfg = tiny_llama().scaled(n_layers=3)
    rng = np.random.default_rng(4)
    prompts = [rng.integers(0, cfg.vocab, 60).tolist()]
    ref = LLMEngine.from_config(cfg, "cpu", EngineConfig(max_model_len=128, max_running=6,
                                                         max_step_tokens=64, prefill_chunk=16,
                                                         prefix_cache=False),
                                source=RandomSource(cfg, seed=5))
    want = [o.token_ids for o in ref.generate(prompts, SamplingParams(max_tokens=9,
                                                                      ignore_eos=True))]
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_async_long_worker, args=(r, 3, port, q)) for r in range(3)]
    for p in procs:
        p.start()
    try:
        got, pipelined = q.get(timeout=240)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert got == want
    assert pipelined >= 2      # chunks 2 and 3 of 4 followed the one before them
