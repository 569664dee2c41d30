"""Failure recovery of the pipeline engines (synchronous and wave-pipelined)
on CPU ranks (gloo): a stage's process dies mid-generation; the survivors re-plan the layers over the
remaining ranks, replay the unfinished requests, and the output equals an
undisturbed single-process run.  The failure is made on the host (a rank
exits); no GPU is involved."""
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cfg():
    from swarmllm_b200.models.config import tiny_llama
    return tiny_llama().scaled(n_layers=4)


def _prompts():
    rng = np.random.default_rng(0)
    return [rng.integers(0, 32000, n).tolist() for n in (12, 7, 20)]


def _worker(rank, world, port, ctl_port, crash_rank, crash_after, q, waves=False):
    import torch
    torch.set_num_threads(1)
    from swarmllm_b200.engine.engine import EngineConfig
    from swarmllm_b200.engine.sampling import SamplingParams
    from swarmllm_b200.models.weights import RandomSource
    from swarmllm_b200.parallel.failover import ResilientPipeline
    from swarmllm_b200.parallel.pipeline import PipelineEngine
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    cfg = _cfg()
    ecfg = EngineConfig(max_model_len=128, max_running=4, max_step_tokens=64, prefill_chunk=64,
                        prefix_cache=False, cuda_graphs=False)

    def build():
        if waves:
            from swarmllm_b200.parallel.async_pipeline import AsyncPipelineEngine
            eng = AsyncPipelineEngine(cfg, ecfg, lambda: RandomSource(cfg, seed=5), "cpu")
            if rank == crash_rank:
                steps = {"n": 0}
                real_run = eng.run

                def run(on_events=None, stop_when=None, on_step=None):
                    def hook():
                        steps["n"] += 1
                        if steps["n"] > crash_after:
                            os._exit(17)  # the process dies between its wave steps
                        if on_step is not None:
                            on_step()
                    return real_run(on_events, stop_when, hook)
                eng.run = run
            return eng
        eng = PipelineEngine(cfg, ecfg, lambda: RandomSource(cfg, seed=5), "cpu")
        if rank == crash_rank:
            steps = {"n": 0}
            real = eng.step

            def step():
                steps["n"] += 1
                if steps["n"] > crash_after:
                    os._exit(17)  # the process dies between steps
                return real()
            eng.step = step
        return eng

    # grace well above the group timeout: a survivor that learns of the failure
    # only from its own group timeout must still register on a loaded machine;
    # the timeout itself stays above a step's time when the host is busy (a
    # healthy step that overruns it would be taken for a second failure)
    rp = ResilientPipeline(build, rank, world, "127.0.0.1", ctl_port, pg_timeout_s=10.0,
                           grace_s=25.0)
    out = rp.generate(_prompts(), SamplingParams(max_tokens=10, ignore_eos=True))
    if rank == 0:
        q.put((out, rp.recoveries, rp.members))
    rp.close()


def _waves_worker(rank, world, port, ctl_port, crash_rank, crash_after, q):
    _worker(rank, world, port, ctl_port, crash_rank, crash_after, q, waves=True)


@pytest.mark.parametrize("waves", [False, True])
def test_stage_failure_replans_and_replays(waves):
    from swarmllm_b200.engine import EngineConfig, LLMEngine, SamplingParams
    from swarmllm_b200.models.weights import RandomSource
    cfg = _cfg()
    ref = LLMEngine.from_config(cfg, "cpu", EngineConfig(max_model_len=128, max_running=4,
                                                         max_step_tokens=64, prefill_chunk=64,
                                                         prefix_cache=False),
                                source=RandomSource(cfg, seed=5))
    want = [o.token_ids for o in ref.generate(_prompts(), SamplingParams(max_tokens=10,
                                                                        ignore_eos=True))]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port, ctl = _free_port(), _free_port()
    fn = _waves_worker if waves else _worker
    procs = [ctx.Process(target=fn, args=(r, 3, port, ctl, 2, 4, q)) for r in range(3)]
    for p in procs:
        p.start()
    try:
        out, recoveries, members = q.get(timeout=240)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert procs[2].exitcode == 17
    assert procs[0].exitcode == 0 and procs[1].exitcode == 0
    assert recoveries == 1 and members == [0, 1]
    assert out == want


def test_outlier_tracker_ejects_repeat_failures():
    from swarmllm_b200.parallel.failover import OutlierTracker
    now = [0.0]
    t = OutlierTracker(limit=2, window_s=10.0, eject_s=100.0, clock=lambda: now[0])
    t.record(3)
    assert t.ejected() == set() and t.members([0, 1, 3]) == [0, 1, 3]
    now[0] = 20.0                       # the first failure left the window
    t.record(3)
    assert t.ejected() == set()
    now[0] = 25.0
    t.record(3)                         # two inside the window: ejected
    assert t.ejected() == {3} and t.members([0, 1, 3]) == [0, 1]
    now[0] = 126.0                      # cool-down over
    assert t.ejected() == set() and t.members([0, 1, 3]) == [0, 1, 3]
    t2 = OutlierTracker(limit=1, clock=lambda: now[0])
    t2.record(0)
    assert t2.members([0]) == [0]       # never an empty membership
