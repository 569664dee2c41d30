"""Request-level data parallelism (parallel/replicas.py): CPU engine replicas
in their own processes behind one front scheduler."""
import asyncio

import numpy as np
import pytest

pytestmark = pytest.mark.timeout(600)


def _spec():
    from swarmllm_b200.engine import EngineConfig
    from swarmllm_b200.models.config import tiny_llama
    cfg = tiny_llama()
    ecfg = EngineConfig(max_model_len=160, max_running=8, max_step_tokens=256, prefill_chunk=64)
    return cfg, {"cfg": cfg, "device": "cpu", "ecfg": ecfg, "seed": 3}


def _bad_factory(spec, idx):
    from swarmllm_b200.parallel.replicas import engine_factory
    if idx == 1:
        raise RuntimeError("replica 1 has no device")
    return engine_factory(spec, idx)


def test_replicas_match_one_engine_and_share_the_work():
    from swarmllm_b200.engine import LLMEngine, SamplingParams
    from swarmllm_b200.parallel.replicas import ReplicaSet
    cfg, spec = _spec()
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, cfg.vocab, n).tolist() for n in (9, 30, 17, 5, 22, 12)]
    sp = SamplingParams(max_tokens=8, ignore_eos=True)
    want = [o.token_ids for o in LLMEngine.from_config(cfg, "cpu", spec["ecfg"], seed=3)
            .generate(prompts, sp)]
    rs = ReplicaSet(cfg, spec, 2)
    try:
        outs = rs.generate(prompts, sp)
        assert [o.token_ids for o in outs] == want
        assert {o.replica for o in outs} == {0, 1}          # both replicas served
        assert rs.sched.num_running == 0 and rs.bm.num_pages > 0 and rs.steps > 0
    finally:
        rs.close()


def test_prefix_affinity_and_slack():
    from swarmllm_b200.engine import SamplingParams
    from swarmllm_b200.parallel.replicas import ReplicaSet
    cfg, spec = _spec()
    rng = np.random.default_rng(1)
    shared = rng.integers(0, cfg.vocab, 64).tolist()
    sp = SamplingParams(max_tokens=4, ignore_eos=True)
    rs = ReplicaSet(cfg, spec, 2, affinity_tokens=64, slack=10_000)
    try:
        a = rs.add_request(shared + [1, 2], sp)
        b = rs.add_request(rng.integers(0, cfg.vocab, 70).tolist(), sp)   # other prefix
        assert rs.reqs[a].replica != rs.reqs[b].replica
        while rs.has_work():                           # a's pages are cached once it is done
            rs.step(0.1)
        c = rs.add_request(shared + [3], sp)          # same prefix: same replica as a
        assert rs.reqs[c].replica == rs.reqs[a].replica
        while rs.has_work():
            rs.step(0.1)
        assert rs.bm.prefix_hit_tokens > 0             # c reused a's cached pages
        rs.slack = 0                                   # now load wins over affinity
        e = rs.add_request(rng.integers(0, cfg.vocab, 100).tolist(), sp)
        d = rs.add_request(shared + [4], sp)
        assert rs.reqs[d].replica != rs.reqs[e].replica
        while rs.has_work():
            rs.step(0.1)
    finally:
        rs.close()


def test_a_failed_replica_is_left_out():
    from swarmllm_b200.engine import SamplingParams
    from swarmllm_b200.parallel.replicas import ReplicaSet
    cfg, spec = _spec()
    rs = ReplicaSet(cfg, spec, 2, factory=_bad_factory)
    try:
        assert 1 in rs.dead and "no device" in rs.dead[1]
        outs = rs.generate([[1, 2, 3], [4, 5, 6, 7]], SamplingParams(max_tokens=3,
                                                                     ignore_eos=True))
        assert all(o.replica == 0 and len(o.token_ids) == 3 for o in outs)
    finally:
        rs.close()


def test_async_server_loop_over_replicas():
    """The HTTP server's engine loop drives a replica set like one engine."""
    from swarmllm_b200.engine import SamplingParams
    from swarmllm_b200.parallel.replicas import ReplicaSet
    from swarmllm_b200.serve.api import AsyncEngine
    cfg, spec = _spec()
    rs = ReplicaSet(cfg, spec, 2)
    ae = AsyncEngine(rs)

    async def one(prompt):
        rid, q = ae.submit(prompt, SamplingParams(max_tokens=5, ignore_eos=True))
        toks = []
        while True:
            m = await q.get()
            if m[0] == "token":
                toks.append(m[1])
            elif m[0] == "done":
                return toks, m[2].route
            else:
                raise AssertionError(m)

    async def main():
        return await asyncio.gather(*(one([7, 8, 9 + i]) for i in range(4)))
    try:
        res = asyncio.run(main())
        assert all(len(t) == 5 for t, _ in res)
        assert {r for _, r in res} == {"replica0", "replica1"}
    finally:
        ae.shutdown()
        rs.close()


def test_http_server_over_replicas():
    """The OpenAI route and the status route over a replica set."""
    import socket
    import threading
    import time

    import requests
    import uvicorn

    from swarmllm_b200.parallel.replicas import ReplicaSet
    from swarmllm_b200.serve.api import AsyncEngine, create_app
    from swarmllm_b200.serve.tokenizer import ByteTokenizer
    cfg, spec = _spec()
    rs = ReplicaSet(cfg, spec, 2)
    ae = AsyncEngine(rs)
    app = create_app(ae, ByteTokenizer(cfg.vocab), "tiny", max_model_len=160)
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    srv = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="error"))
    th = threading.Thread(target=srv.run, daemon=True)
    th.start()
    try:
        for _ in range(200):
            if srv.started:
                break
            time.sleep(0.05)
        url = f"http://127.0.0.1:{port}"
        r = requests.post(url + "/v1/completions", json={"model": "tiny", "prompt": "hello there",
                                                         "max_tokens": 6, "temperature": 0},
                          timeout=120)
        assert r.status_code == 200, r.text
        assert r.json()["usage"]["completion_tokens"] == 6
        st = requests.get(url + "/api/status", timeout=30).json()
        assert st["kv_pages"] > 0 and st["steps"] > 0 and st["ready"]
    finally:
        srv.should_exit = True
        th.join(5)
        ae.shutdown()
        rs.close()


def _flaky_factory(spec, idx):
    """Replica 1's engine fails on its third step (a stand-in for a device
    error); replica 0 is healthy."""
    from swarmllm_b200.parallel.replicas import engine_factory
    eng = engine_factory(spec, idx)
    if idx == 1:
        real, n = eng.step, [0]

        def step():
            n[0] += 1
            if n[0] >= 3:
                raise RuntimeError("device lost")
            return real()
        eng.step = step
    return eng


def test_a_replica_failing_mid_run_fails_only_its_requests():
    from swarmllm_b200.engine import SamplingParams
    from swarmllm_b200.parallel.replicas import ReplicaSet
    cfg, spec = _spec()
    rs = ReplicaSet(cfg, spec, 2, factory=_flaky_factory)
    try:
        sp = SamplingParams(max_tokens=6, ignore_eos=True)
        rids = [rs.add_request([1, 2, 3 + i], sp) for i in range(4)]
        on = {rid: rs.reqs[rid].replica for rid in rids}
        assert set(on.values()) == {0, 1}
        done = {}
        while rs.has_work():
            for rid, tok, fin in rs.step(0.1):
                if fin:
                    done[rid] = tok
        for rid in rids:
            if on[rid] == 1:
                assert done[rid] is None and "device lost" in rs.error_of(rid)
            else:
                assert rs.error_of(rid) is None and len(rs.output(rid)) == 6
        assert 1 in rs.dead
        late = rs.generate([[9, 9, 9]], sp)          # new work goes to the survivor
        assert late[0].replica == 0 and len(late[0].token_ids) == 6
    finally:
        rs.close()
