"""CPU tests: quant formats, GGUF read/write + shard layout, block manager,
scheduler, planner, draft tree, config loading."""
import numpy as np
import pytest

from swarmllm_b200.gguf import quants as Q


@pytest.mark.parametrize("qt", [Q.Q4_0, Q.Q8_0, Q.Q4_K, Q.Q6_K, Q.IQ4_NL, Q.IQ4_XS, Q.MXFP4,
                                Q.F16, Q.BF16, Q.F32])
def test_quant_roundtrip(qt):
    rng = np.random.default_rng(qt)
    x = rng.standard_normal((3, 512)).astype(np.float32) * 0.02
    b = Q.quantize(x, qt)
    assert b.shape == (3, Q.nbytes(qt, 512))
    y = Q.dequantize(b, qt)
    tol = {Q.MXFP4: 0.25, Q.Q4_0: 0.15, Q.IQ4_NL: 0.15, Q.IQ4_XS: 0.15, Q.Q4_K: 0.06, Q.Q6_K: 0.03}.get(qt, 0.005)
    assert np.abs(y - x).max() <= tol * np.abs(x).max()
    # dequantize(quantize(dequantize(b))) is a fixed point for the exact formats
    if qt in (Q.Q8_0, Q.F16, Q.F32, Q.BF16):
        assert np.array_equal(Q.quantize(y, qt), b)


def test_q4k_layout_against_definition():
    """Hand-built Q4_K block: d=1, dmin=0.5, sc_j=j+1, m_j=2j, codes = position % 16."""
    sc = np.arange(1, 9)[None]
    m = (2 * np.arange(8))[None]
    q = (np.arange(256) % 16).astype(np.uint8)[None]
    qs = np.zeros((1, 128), np.uint8)
    for g in range(4):
        qs[:, 32 * g:32 * g + 32] = q[:, 64 * g:64 * g + 32] | (q[:, 64 * g + 32:64 * g + 64] << 4)
    blk = np.concatenate([np.array([1.0], np.float16).view(np.uint8)[None],
                          np.array([0.5], np.float16).view(np.uint8)[None],
                          Q._pack_q4k_scales(sc, m), qs], 1)
    y = Q.dequantize(blk, Q.Q4_K)[0]
    for k in range(256):
        j = k // 32
        assert y[k] == pytest.approx((j + 1) * (k % 16) - 0.5 * (2 * j))


def test_q4k_repack_host_permutation():
    rng = np.random.default_rng(0)
    b = Q.quantize(rng.standard_normal((128, 512)).astype(np.float32), Q.Q4_K)
    packed = Q.q4k_repack_host(b, 128, 512)
    assert packed.shape == (1, 2, 128, 144)
    # word 0 of row 0, superblock 0: nibble p holds k = perm[p]
    vals = np.zeros(8, np.int64)
    w = packed[0, 0, 0, :4].view(np.uint32)[0]
    for p in range(8):
        vals[p] = (w >> (4 * p)) & 15
    src = b.reshape(128, 2, 144)[0, 0, 16:]
    codes = [(src[k] & 15) for k in range(8)]
    assert list(vals) == [codes[i] for i in (0, 2, 4, 6, 1, 3, 5, 7)]


def test_gguf_write_read_and_shards(tmp_path):
    from swarmllm_b200.gguf.file import GGUFReader, ShardedGguf, write_sharded
    from swarmllm_b200.models.config import from_gguf_metadata, tiny_llama
    from swarmllm_b200.models.weights import tensor_specs, write_random_gguf
    cfg = tiny_llama()
    path = str(tmp_path / "m.gguf")
    write_random_gguf(cfg, path, seed=5)
    r = GGUFReader(path)
    assert r.metadata["general.architecture"] == "llama"
    assert from_gguf_metadata(r.metadata) == cfg
    names = {n for n, _, _ in tensor_specs(cfg)}
    assert set(r.tensors) == names
    ti = r.tensors["blk.0.attn_q.weight"]
    assert ti.shape == (cfg.q_dim, cfg.hidden) and ti.qtype == Q.Q4_0
    w = r.tensor_float("blk.1.ffn_down.weight")
    assert w.shape == (cfg.hidden, cfg.ffn) and 0.01 < w.std() < 0.03
    d = str(tmp_path / "shards")
    write_sharded(path, d, layers_per_shard=1)
    s = ShardedGguf(d)
    for n in ("token_embd.weight", "blk.1.attn_k.weight", "output.weight"):
        assert np.array_equal(s.tensor_bytes(n), np.asarray(r.tensor_bytes(n)))
    # a corrupted shard fails its checksum
    import glob
    f = sorted(glob.glob(d + "/shard_*.bin"))[0]
    with open(f, "r+b") as fh:
        fh.seek(10)
        fh.write(b"\xff\xff")
    with pytest.raises(IOError):
        ShardedGguf(d)


def test_block_manager_prefix_sharing_and_truncate():
    from swarmllm_b200.utils.ext import native
    bm = native().BlockManager(16, 4, True)
    toks = list(range(10))
    assert bm.add_sequence(1, toks) == 0
    slots = bm.append_slots(1, 10)
    assert len(slots) == 10 and bm.num_free() == 13
    bm.commit_tokens(1, toks)
    bm.free_sequence(1)
    assert bm.num_free() == 16 and bm.num_cached_pages == 2  # 2 full pages cached
    # same prefix: first 2 pages (8 tokens) shared
    assert bm.add_sequence(2, toks + [99]) == 8
    assert bm.prefix_hit_tokens == 8
    s2 = bm.append_slots(2, 3)
    assert len(s2) == 3
    bm.truncate(2, 9)
    assert bm.seq_len(2) == 9
    t = bm.block_table([2], 8)
    assert t.shape == (1, 8)
    # fork shares pages; the partial last page is copied
    src, dst = bm.fork(2, 3)
    assert src >= 0 and dst >= 0 and src != dst


def test_scheduler_chunked_prefill_and_preemption():
    from swarmllm_b200.utils.ext import native
    N = native()
    bm = N.BlockManager(12, 4, False)
    s = N.Scheduler(bm, 8, 4, 6)
    s.add_request(1, list(range(10)), 5, -1)
    s.add_request(2, list(range(3)), 5, -1)
    p = s.schedule()
    assert list(p.seq_ntok) == [6, 2] and list(p.seq_sample) == [0, 0]
    s.commit(p, [])
    p = s.schedule()
    # seq 1 finishes prefill (4 tokens), seq 2 finishes prefill (1 token)
    assert sorted(p.seq_ntok) == [1, 4] and list(p.seq_sample) == [1, 1]
    s.commit(p, [7, 8])
    steps, done = 0, set()
    while s.has_work() and steps < 50:
        p = s.schedule()
        done |= set(s.commit(p, [3] * int(sum(p.seq_sample))))
        steps += 1
    assert done == {1, 2}
    assert len(s.output(1)) == 5 and len(s.output(2)) == 5


def test_planner_bottleneck_and_route():
    from swarmllm_b200.utils.ext import native
    N = native()
    plan = N.plan_bottleneck([1.0] * 10, [], [1.0, 1.0], [], 0.0)
    assert plan.feasible and list(plan.first_layer) == [0, 5, 10]
    plan = N.plan_bottleneck([1.0] * 10, [1.0] * 10, [1.0, 1.0, 1.0], [4, 4, 4], 0.0)
    assert plan.feasible and max(np.diff(plan.first_layer)) <= 4
    plan = N.plan_bottleneck([1.0] * 10, [1.0] * 10, [1.0, 1.0], [4, 4], 0.0)
    assert not plan.feasible
    # a faster device takes more layers
    plan = N.plan_bottleneck([1.0] * 12, [], [2.0, 1.0], [], 0.0)
    assert plan.first_layer[1] == 8
    p, devs = N.plan_route([1.0] * 8, [1.0] * 8, [1.0, 1.0, 1.0], [8, 4, 4], [1.0, 1.0, 1.0], 5.0)
    assert p.feasible and devs == [0]  # hop cost makes one device best
    p, devs = N.plan_route([1.0] * 8, [1.0] * 8, [1.0, 1.0, 1.0], [4, 4, 4], [1.0, 1.0, 1.0], 0.1)
    assert p.feasible and len(devs) == 2


def test_draft_tree_expand_and_walk():
    from swarmllm_b200.utils.ext import native
    t = native().DraftTree(100, 64)
    f = t.expand([5, 6, 7], [-0.1, -1.0, -2.0], 3, 2)
    assert f == [1, 2] and t.tokens()[1:] == [5, 6]
    f = t.expand([8, 9, 10, 11], [-0.1, -0.5, -0.2, -3.0], 2, 3)
    assert len(f) == 3 and all(t.depths()[i] == 2 for i in f)
    masks = t.masks()
    assert masks[0] == 1 and all(masks[i] & 1 for i in range(len(t)))
    # target picks 5 at root, then the child of node 1 with token 8, then stops
    tgt = [5, 8] + [0] * (len(t) - 2)
    n8 = t.tokens().index(8)
    tgt[n8] = 42
    path, bonus = t.walk(tgt)
    assert path == [0, 1, n8] and bonus == 42


def test_config_env_and_toml(tmp_path):
    from swarmllm_b200.utils.config import load_engine_config
    p = tmp_path / "c.toml"
    p.write_text("[inference]\nprefill_chunk_tokens = 128\nmax_concurrent_decode_batch = 7\n")
    c = load_engine_config(str(p), env={"SWARMLLM_MAX_MODEL_LEN": "999", "SWARMLLM_CUDA_GRAPH": "0"})
    assert c.prefill_chunk == 128 and c.max_running == 7 and c.max_model_len == 999
    assert c.cuda_graphs is False


def test_rope_scaling_llama3_matches_definition():
    from swarmllm_b200.models.config import llama33_70b, rope_inv_freq
    inv, f = rope_inv_freq(llama33_70b())
    assert f == 1.0 and len(inv) == 64
    base = 1.0 / (500000.0 ** (np.arange(0, 128, 2) / 128))
    assert inv[0] == pytest.approx(base[0])         # high frequency untouched
    assert inv[-1] == pytest.approx(base[-1] / 8)   # low frequency divided by the factor
