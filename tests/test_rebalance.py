"""Stage rebalancing (CPU): measured stage times re-weight the layer costs and
move layers off a slow stage; over gloo ranks the wave-pipelined engine is
rebuilt with the new cut between requests and still gives single-process
output."""
import multiprocessing as mp
import os
import socket

import numpy as np

from swarmllm_b200.parallel.rebalance import StageRebalancer


def test_rebalancer_moves_layers_off_a_slow_stage():
    r = StageRebalancer([1.0] * 8, threshold=0.1)
    # stage 0 (layers 0-3) measured twice as slow as stage 1
    new = r.propose([0, 4, 8], [8.0, 4.0])
    assert new is not None and new[1] < 4
    # balanced stages: no move
    assert StageRebalancer([1.0] * 8).propose([0, 4, 8], [4.0, 4.1]) is None


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, ctl_port, q):
    import torch
    torch.set_num_threads(1)
    from swarmllm_b200.engine.engine import EngineConfig
    from swarmllm_b200.engine.sampling import SamplingParams
    from swarmllm_b200.models.config import tiny_llama
    from swarmllm_b200.models.weights import RandomSource
    from swarmllm_b200.parallel.async_pipeline import AsyncPipelineEngine
    from swarmllm_b200.parallel.failover import ResilientPipeline
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    cfg = tiny_llama().scaled(n_layers=4)
    ecfg = EngineConfig(max_model_len=128, max_running=4, max_step_tokens=64, prefill_chunk=64,
                        prefix_cache=False, cuda_graphs=False)

    def build(bounds=None):
        return AsyncPipelineEngine(cfg, ecfg, lambda: RandomSource(cfg, seed=5), "cpu",
                                   bounds=bounds)
    rp = ResilientPipeline(build, rank, world, "127.0.0.1", ctl_port, pg_timeout_s=20.0)
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, cfg.vocab, n).tolist() for n in (9, 14)]
    sp = SamplingParams(max_tokens=6, ignore_eos=True)
    out1 = rp.generate(prompts, sp)
    before = list(rp.eng.bounds)
    moved = rp.rebalance(StageRebalancer([1.0] * 4), stage_s=[3.0, 1.0])  # stage 0 slow
    after = list(rp.eng.bounds)
    out2 = rp.generate(prompts, sp)
    if rank == 0:
        q.put((out1, out2, moved, before, after))
    rp.close()


def test_rebalance_rebuilds_wave_pipeline_with_same_output():
    from swarmllm_b200.engine import EngineConfig, LLMEngine, SamplingParams
    from swarmllm_b200.models.config import tiny_llama
    from swarmllm_b200.models.weights import RandomSource
    cfg = tiny_llama().scaled(n_layers=4)
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, cfg.vocab, n).tolist() for n in (9, 14)]
    ref = LLMEngine.from_config(cfg, "cpu", EngineConfig(max_model_len=128, max_running=4,
                                                         max_step_tokens=64, prefill_chunk=64,
                                                         prefix_cache=False),
                                source=RandomSource(cfg, seed=5))
    want = [o.token_ids for o in ref.generate(prompts, SamplingParams(max_tokens=6,
                                                                      ignore_eos=True))]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port, ctl = _free_port(), _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, ctl, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        out1, out2, moved, before, after = q.get(timeout=240)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert moved and after[1] < before[1]
    assert out1 == want and out2 == want
