"""Prefix-KV snapshots: export from one engine, import into another (same
process, bytes round trip, and between two gloo ranks)."""
import os
import socket
from datetime import timedelta

import pytest
import torch


def _engine(seed=5, pages=0):
    from swarmllm_b200.engine import EngineConfig, LLMEngine
    from swarmllm_b200.models.config import tiny_llama
    from swarmllm_b200.models.weights import RandomSource
    cfg = tiny_llama()
    ec = EngineConfig(max_model_len=256, max_running=4, max_step_tokens=256, prefill_chunk=256)
    if pages:
        ec.num_pages = pages
    return LLMEngine.from_config(cfg, "cpu", ec, source=RandomSource(cfg, seed=seed))


PROMPT = list(range(3, 3 + 70))   # 4 full 16-token pages + 6 tokens


def _gen(eng, prompt, n=6):
    from swarmllm_b200.engine import SamplingParams
    return eng.generate([prompt], SamplingParams(max_tokens=n))[0].token_ids


def test_export_import_same_output_and_prefix_hit():
    from swarmllm_b200.engine.prefix_share import PrefixSnapshot
    a = _engine()
    out_a = _gen(a, PROMPT)
    snap = a.export_prefix(PROMPT)
    assert snap is not None and snap.n_pages == 4 and snap.tokens == PROMPT[:64]
    snap2 = PrefixSnapshot.from_bytes(snap.to_bytes())
    assert torch.equal(snap2.kv, snap.kv) and snap2.tokens == snap.tokens
    b = _engine()
    assert b.import_prefix(snap2) == 64
    assert b.import_prefix(snap2) == 0            # already cached: nothing new
    hits0 = b.bm.prefix_hit_tokens
    out_b = _gen(b, PROMPT)
    assert out_b == out_a
    assert b.bm.prefix_hit_tokens - hits0 == 64   # the prompt's 4 full pages came from the snapshot


def test_import_rejects_other_geometry_or_model():
    a = _engine()
    _gen(a, PROMPT)
    snap = a.export_prefix(PROMPT)
    from swarmllm_b200.engine.prefix_share import PrefixSnapshot
    bad = PrefixSnapshot("other-model", snap.tokens, snap.page_size, snap.kv)
    with pytest.raises(ValueError):
        _engine().import_prefix(bad)
    bad = PrefixSnapshot(snap.model, snap.tokens, snap.page_size, snap.kv[:, :, :, :1])
    with pytest.raises(ValueError):
        _engine().import_prefix(bad)


def test_nothing_cached_exports_none():
    assert _engine().export_prefix(PROMPT) is None


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, port, q):
    import torch.distributed as dist
    from swarmllm_b200.engine.prefix_share import recv_prefix, send_prefix
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=timedelta(seconds=60))
    try:
        eng = _engine()
        if rank == 0:
            out = _gen(eng, PROMPT)
            send_prefix(eng.export_prefix(PROMPT), 1)
            dist.send(torch.tensor(out), 1)
        else:
            snap = recv_prefix(0)
            ref = torch.zeros(6, dtype=torch.int64)
            dist.recv(ref, 0)
            n = eng.import_prefix(snap)
            hits0 = eng.bm.prefix_hit_tokens
            out = _gen(eng, PROMPT)
            q.put((n, eng.bm.prefix_hit_tokens - hits0, out == ref.tolist()))
    finally:
        dist.destroy_process_group()


def test_snapshot_between_gloo_ranks():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=180)
        assert p.exitcode == 0
    n, hits, same = q.get(timeout=5)
    assert n == 64 and hits == 64 and same


@pytest.mark.gpu
def test_export_import_gpu_engine():
    from swarmllm_b200.engine import EngineConfig, LLMEngine
    from swarmllm_b200.models.config import tiny_llama
    from swarmllm_b200.models.weights import RandomSource
    from swarmllm_b200.engine.prefix_share import PrefixSnapshot
    cfg = tiny_llama()
    ec = EngineConfig(max_model_len=256, max_running=4, max_step_tokens=256, prefill_chunk=256,
                      graph_sizes=(1, 2, 4))
    mk = lambda: LLMEngine.from_config(cfg, "cuda:0", ec, source=RandomSource(cfg, seed=5))
    a = mk()
    out_a = _gen(a, PROMPT)
    snap = PrefixSnapshot.from_bytes(a.export_prefix(PROMPT).to_bytes())
    b = mk()
    assert b.import_prefix(snap) == 64
    hits0 = b.bm.prefix_hit_tokens
    assert _gen(b, PROMPT) == out_a
    assert b.bm.prefix_hit_tokens - hits0 == 64


def test_persisted_cache_reloads_and_stamp_mismatch_discards(tmp_path):
    a = _engine()
    out_a = _gen(a, PROMPT)
    _gen(a, PROMPT[:40])                       # a prefix of the first: saved inside it
    path = str(tmp_path / "kv.bin")
    assert a.save_prefix_cache(path) == 64
    b = _engine()
    assert b.load_prefix_cache(path) == 64
    hits0 = b.bm.prefix_hit_tokens
    assert _gen(b, PROMPT) == out_a
    assert b.bm.prefix_hit_tokens - hits0 == 64
    c = _engine()
    c.cfg.name = "another-model"               # another model: the stamp differs
    assert c.load_prefix_cache(path) == 0 and c.bm.num_cached_pages == 0
    assert _engine().load_prefix_cache(str(tmp_path / "missing.bin")) == 0


def test_cache_salt_separates_namespaces():
    from swarmllm_b200.engine.engine import cache_salt
    from swarmllm_b200.utils.ext import native
    N = native()
    bm = N.BlockManager(64, 16, True)
    toks = list(range(100, 150))
    assert bm.add_sequence(1, toks) == 0
    bm.append_slots(1, len(toks))
    bm.commit_tokens(1, toks)
    bm.free_sequence(1)
    s = cache_salt("adapter-a")
    assert s != 0 and s != cache_salt("adapter-b") and cache_salt(None) == 0
    assert bm.add_sequence(2, toks, s) == 0           # other namespace: no hit
    assert bm.add_sequence(3, toks) == 48              # base namespace: 3 pages hit
    assert len(bm.cached_prefix_pages(toks)) == 3 and len(bm.cached_prefix_pages(toks, s)) == 0
