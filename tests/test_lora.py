"""LoRA adapters: GGUF round trip, the CPU oracle against merged weights, and
the GPU per-row application (mixed adapters in one batch) against the oracle."""
import numpy as np
import pytest
import torch

DEV = "cuda:0"


def _cfg(qt="Q8_0", layers=2):
    from swarmllm_b200.models.config import ModelConfig
    return ModelConfig(name="t", arch="llama", n_layers=layers, hidden=512, n_heads=8, n_kv_heads=2,
                       head_dim=64, ffn=1024, vocab=1024, weight_qtype=qt, embed_qtype="F16",
                       output_qtype=qt)


def _batch(tokens, positions, bt, device, sample_rows, lora_ids=None):
    from swarmllm_b200.models.llama import StepBatch
    t = lambda a, dt=torch.int32: torch.as_tensor(np.asarray(a), dtype=dt, device=device)
    b = StepBatch(t(tokens), t(positions), t(positions), t(bt), t(np.asarray(positions) + 1),
                  t(sample_rows, torch.int64), 256)
    if lora_ids is not None:
        b.lora_ids = t(lora_ids)
    return b


def test_lora_gguf_round_trip(tmp_path):
    from swarmllm_b200.models.lora import LoraAdapter
    ad = LoraAdapter.random(_cfg(), rank=4, seed=1, alpha=8.0)
    p = str(tmp_path / "a.gguf")
    ad.write_gguf(p)
    back = LoraAdapter.from_gguf(p, "x")
    assert back.alpha == 8.0 and set(back.tensors) == set(ad.tensors)
    for k, (a, b) in ad.tensors.items():
        np.testing.assert_array_equal(back.tensors[k][0], a)
        np.testing.assert_array_equal(back.tensors[k][1], b)
        assert back.scale(k) == 2.0


def test_cpu_lora_equals_merged_weights():
    """The oracle's per-row delta equals running with W + scale * B A merged."""
    from swarmllm_b200.models.llama import LlamaCPU
    from swarmllm_b200.models.lora import LoraAdapter
    from swarmllm_b200.models.weights import RandomSource
    from swarmllm_b200.ops.attention import PagedKVCache
    cfg = _cfg()
    src = RandomSource(cfg, seed=3)
    ad = LoraAdapter.random(cfg, rank=8, seed=2, alpha=16.0)
    m = LlamaCPU(cfg, src)
    m.lora_adapters = [ad]
    merged = LlamaCPU(cfg, src)
    names = {"attn_q": "wq", "attn_k": "wk", "attn_v": "wv", "attn_output": "wo",
             "ffn_gate": "wg", "ffn_up": "wu", "ffn_down": "wd"}
    for base, (a, b) in ad.tensors.items():
        _, layer, suffix, _ = base.split(".")
        L = merged.layers[int(layer)]
        w = getattr(L, names[suffix])
        setattr(L, names[suffix], w + ad.scale(base) * torch.from_numpy(b @ a))
    rng = np.random.default_rng(0)
    toks = rng.integers(0, cfg.vocab, 12)
    pos = np.arange(12)
    bt = np.tile(np.arange(8, dtype=np.int32), (12, 1))
    kv = lambda: PagedKVCache(cfg.n_layers, 8, cfg.n_kv_heads, cfg.head_dim, "cpu", dtype=torch.float32)
    la = m.forward(_batch(toks, pos, bt, "cpu", [11], lora_ids=[0] * 12), kv())
    lb = merged.forward(_batch(toks, pos, bt, "cpu", [11]), kv())
    lc = m.forward(_batch(toks, pos, bt, "cpu", [11], lora_ids=[-1] * 12), kv())
    torch.testing.assert_close(la, lb, rtol=1e-4, atol=1e-4)
    assert float((la - lc).abs().max()) > 1e-2   # the adapter changes the output


def test_cpu_engine_lora_requests():
    from swarmllm_b200.engine import EngineConfig, LLMEngine, SamplingParams
    from swarmllm_b200.models.lora import LoraAdapter
    from swarmllm_b200.models.weights import RandomSource
    cfg = _cfg()
    ec = EngineConfig(max_model_len=64, max_running=4, max_step_tokens=64, prefill_chunk=64,
                      max_loras=2)
    eng = LLMEngine.from_config(cfg, "cpu", ec, source=RandomSource(cfg, seed=5))
    eng.load_lora(LoraAdapter.random(cfg, rank=8, seed=4, std=0.3), "a")
    p = list(range(1, 17))
    sp = SamplingParams(max_tokens=6)
    r0 = eng.add_request(p, sp)
    r1 = eng.add_request(p, sp, lora="a")
    out = {}
    while eng.has_work():
        for rid, tok, fin in eng.step():
            out.setdefault(rid, []).append(tok)
    base = LLMEngine.from_config(cfg, "cpu", EngineConfig(max_model_len=64, max_running=4,
                                                          max_step_tokens=64, prefill_chunk=64),
                                 source=RandomSource(cfg, seed=5)).generate([p], sp)[0].token_ids
    assert out[r0] == base
    assert out[r1] != base


@pytest.mark.gpu
@pytest.mark.parametrize("qt", ["Q4_K", "Q8_0"])
def test_gpu_lora_rows_match_cpu_oracle(qt):
    """One batch with rows on adapter 0, adapter 1 and no adapter."""
    from swarmllm_b200.models.llama import LlamaCPU, LlamaGPU
    from swarmllm_b200.models.lora import LoraAdapter
    from swarmllm_b200.models.weights import RandomSource
    from swarmllm_b200.ops.attention import PagedKVCache
    cfg = _cfg(qt)
    src = RandomSource(cfg, seed=3)
    ads = [LoraAdapter.random(cfg, rank=8, seed=11, alpha=16.0, name="a"),
           LoraAdapter.random(cfg, rank=16, seed=12, targets=("attn_q", "attn_v", "ffn_down"),
                              name="b")]
    gpu = LlamaGPU(cfg, src, DEV)
    gpu.enable_lora(max_adapters=2, max_rank=16)
    for a in ads:
        gpu.lora.add(a)
    cpu = LlamaCPU(cfg, src)
    cpu.lora_adapters = ads
    ctx = gpu.make_context(64, 64, 256)
    kvg = PagedKVCache(cfg.n_layers, 8, cfg.n_kv_heads, cfg.head_dim, DEV)
    kvc = PagedKVCache(cfg.n_layers, 8, cfg.n_kv_heads, cfg.head_dim, "cpu", dtype=torch.float32)
    rng = np.random.default_rng(0)
    T = 36
    toks = rng.integers(0, cfg.vocab, T)
    pos = np.arange(T)
    ids = np.array([0] * 12 + [1] * 12 + [-1] * 12, np.int32)
    rows = list(range(T))
    bt = np.tile(np.arange(8, dtype=np.int32), (T, 1))
    lg = gpu.forward(_batch(toks, pos, bt, DEV, rows, ids), kvg, ctx).cpu().double()
    lc = cpu.forward(_batch(toks, pos, bt, "cpu", rows, ids), kvc).double()
    cos = torch.nn.functional.cosine_similarity(lg, lc, dim=-1)
    assert float(cos.min()) > 0.999, cos
    base = cpu.forward(_batch(toks, pos, bt, "cpu", rows, [-1] * T),
                       PagedKVCache(cfg.n_layers, 8, cfg.n_kv_heads, cfg.head_dim, "cpu",
                                    dtype=torch.float32)).double()
    # every adapter visibly changes its rows
    assert float((lc[:24] - base[:24]).abs().max()) > 1e-2


@pytest.mark.gpu
def test_gpu_engine_lora_graphs_and_mixed_batch():
    """Greedy output: adapter requests batched with base requests, CUDA graphs
    on and off agree; base requests are unaffected by adapters in the batch."""
    from swarmllm_b200.engine import EngineConfig, LLMEngine, SamplingParams
    from swarmllm_b200.models.lora import LoraAdapter
    from swarmllm_b200.models.weights import RandomSource
    cfg = _cfg("Q4_K")
    rng = np.random.default_rng(1)
    prompts = [rng.integers(0, cfg.vocab, n).tolist() for n in (9, 30, 17, 44)]
    which = [None, "a", "b", None]
    sp = SamplingParams(max_tokens=10)
    res = []
    for graphs in (False, True):
        ec = EngineConfig(max_model_len=128, max_running=8, max_step_tokens=128, prefill_chunk=64,
                          cuda_graphs=graphs, graph_sizes=(1, 2, 4, 8), max_loras=2, max_lora_rank=8)
        eng = LLMEngine.from_config(cfg, DEV, ec, source=RandomSource(cfg, seed=5))
        eng.load_lora(LoraAdapter.random(cfg, rank=8, seed=21, std=0.3), "a")
        eng.load_lora(LoraAdapter.random(cfg, rank=4, seed=22, std=0.3), "b")
        rid = [eng.add_request(p, sp, lora=w) for p, w in zip(prompts, which)]
        out = {}
        while eng.has_work():
            for r, tok, fin in eng.step():
                out.setdefault(r, []).append(tok)
        res.append([out[r] for r in rid])
    assert res[0] == res[1]
    ec = EngineConfig(max_model_len=128, max_running=8, max_step_tokens=128, prefill_chunk=64,
                      graph_sizes=(1, 2, 4, 8))
    base = LLMEngine.from_config(cfg, DEV, ec, source=RandomSource(cfg, seed=5)).generate(prompts, sp)
    assert res[1][0] == base[0].token_ids and res[1][3] == base[3].token_ids
    assert res[1][1] != base[1].token_ids


@pytest.mark.gpu
def test_gpu_lora_unload_frees_slot():
    """Unloading an adapter zeroes its slot; the next adapter loaded there gives
    the same tokens as an engine that only ever held that adapter."""
    from swarmllm_b200.engine import EngineConfig, LLMEngine, SamplingParams
    from swarmllm_b200.models.lora import LoraAdapter
    from swarmllm_b200.models.weights import RandomSource
    cfg = _cfg("Q4_K")
    prompt = np.random.default_rng(3).integers(0, cfg.vocab, 21).tolist()
    sp = SamplingParams(max_tokens=8)
    ec = EngineConfig(max_model_len=128, max_running=4, max_step_tokens=128, prefill_chunk=64,
                      graph_sizes=(1, 2, 4), max_loras=1, max_lora_rank=8)

    def run(eng, name):
        rid = eng.add_request(prompt, sp, lora=name)
        out = []
        while eng.has_work():
            out += [t for r, t, _ in eng.step() if r == rid]
        eng.release(rid)        # a finished request keeps its adapter until released
        return out
    eng = LLMEngine.from_config(cfg, DEV, ec, source=RandomSource(cfg, seed=5))
    eng.load_lora(LoraAdapter.random(cfg, rank=8, seed=31, std=0.3), "a")
    run(eng, "a")
    assert eng.unload_lora("a") == 0
    eng.load_lora(LoraAdapter.random(cfg, rank=4, seed=32, std=0.3, targets=("attn_q", "ffn_down")), "b")
    got = run(eng, "b")
    ref_eng = LLMEngine.from_config(cfg, DEV, ec, source=RandomSource(cfg, seed=5))
    ref_eng.load_lora(LoraAdapter.random(cfg, rank=4, seed=32, std=0.3, targets=("attn_q", "ffn_down")), "b")
    assert got == run(ref_eng, "b")
