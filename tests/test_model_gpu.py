"""GPU model vs the CPU fp32 oracle, and the GPU engine end to end."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _cfg(qt="Q4_K", layers=2):
    from swarmllm_b200.models.config import ModelConfig
    return ModelConfig(name="t", arch="llama", n_layers=layers, hidden=512, n_heads=8, n_kv_heads=2,
                       head_dim=64, ffn=1024, vocab=1024, weight_qtype=qt, embed_qtype="F16",
                       output_qtype=qt, rope_scaling={"type": "llama3", "factor": 8.0,
                                                      "original_max_position_embeddings": 64})


def _batch(tokens, positions, slots, bt, device, sample_rows):
    from swarmllm_b200.models.llama import StepBatch
    t = lambda a, dt=torch.int32: torch.as_tensor(np.asarray(a), dtype=dt, device=device)
    return StepBatch(t(tokens), t(positions), t(slots), t(bt), t(np.asarray(positions) + 1),
                     t(sample_rows, torch.int64), 256)


@pytest.mark.parametrize("qt", ["Q4_K", "Q8_0", "Q6_K"])
def test_gpu_forward_matches_cpu_oracle(qt):
    from swarmllm_b200.models.llama import LlamaCPU, LlamaGPU
    from swarmllm_b200.models.weights import RandomSource
    from swarmllm_b200.ops.attention import PagedKVCache
    cfg = _cfg(qt)
    src = RandomSource(cfg, seed=3)
    gpu = LlamaGPU(cfg, src, DEV)
    cpu = LlamaCPU(cfg, src)
    ctx = gpu.make_context(64, 8, 256)
    kvg = PagedKVCache(cfg.n_layers, 8, cfg.n_kv_heads, cfg.head_dim, DEV)
    kvc = PagedKVCache(cfg.n_layers, 8, cfg.n_kv_heads, cfg.head_dim, "cpu", dtype=torch.float32)
    rng = np.random.default_rng(0)
    # prefill 40 tokens of one sequence, then 3 decode steps
    toks = rng.integers(0, cfg.vocab, 43)
    bt = np.tile(np.arange(8, dtype=np.int32), (64, 1))
    pos = np.arange(40)
    lg = gpu.forward(_batch(toks[:40], pos, pos, bt[:40], DEV, [39]), kvg, ctx)
    lc = cpu.forward(_batch(toks[:40], pos, pos, bt[:40], "cpu", [39]), kvc)
    cos = torch.nn.functional.cosine_similarity(lg.cpu().double(), lc.double(), dim=-1)
    assert float(cos.min()) > 0.999, cos
    for p in range(40, 43):
        lg = gpu.forward(_batch([toks[p]], [p], [p], bt[:1], DEV, [0]), kvg, ctx)
        lc = cpu.forward(_batch([toks[p]], [p], [p], bt[:1], "cpu", [0]), kvc)
        cos = torch.nn.functional.cosine_similarity(lg.cpu().double(), lc.double(), dim=-1)
        assert float(cos.min()) > 0.999, (p, cos)


def test_engine_graphs_match_eager():
    from swarmllm_b200.engine import EngineConfig, LLMEngine, SamplingParams
    from swarmllm_b200.models.weights import RandomSource
    cfg = _cfg()
    rng = np.random.default_rng(1)
    prompts = [rng.integers(0, cfg.vocab, n).tolist() for n in (5, 37, 64, 100)]
    res = []
    for graphs in (False, True):
        eng = LLMEngine.from_config(cfg, DEV, EngineConfig(max_model_len=256, max_running=8,
                                                           max_step_tokens=128, prefill_chunk=64,
                                                           cuda_graphs=graphs, graph_sizes=(1, 2, 4, 8)),
                                    source=RandomSource(cfg, seed=5))
        outs = eng.generate(prompts, SamplingParams(max_tokens=12))
        res.append([o.token_ids for o in outs])
    assert res[0] == res[1]


def test_engine_gpu_vs_cpu_greedy_tokens():
    """Greedy continuation: GPU and CPU engines agree on (almost) every token."""
    from swarmllm_b200.engine import EngineConfig, LLMEngine, SamplingParams
    from swarmllm_b200.models.weights import RandomSource
    cfg = _cfg("Q8_0")
    rng = np.random.default_rng(2)
    prompts = [rng.integers(0, cfg.vocab, 24).tolist() for _ in range(3)]
    ec = EngineConfig(max_model_len=128, max_running=4, max_step_tokens=128, prefill_chunk=128,
                      graph_sizes=(1, 2, 4))
    g = LLMEngine.from_config(cfg, DEV, ec, source=RandomSource(cfg, seed=7)).generate(
        prompts, SamplingParams(max_tokens=8))
    c = LLMEngine.from_config(cfg, "cpu", ec, source=RandomSource(cfg, seed=7)).generate(
        prompts, SamplingParams(max_tokens=8))
    agree = np.mean([a == b for og, oc in zip(g, c) for a, b in zip(og.token_ids, oc.token_ids)])
    assert agree >= 0.9, (agree, [o.token_ids for o in g], [o.token_ids for o in c])


def _moe_cfg(kind):
    from swarmllm_b200.models.config import ModelConfig
    if kind == "gpt-oss":
        return ModelConfig(name="t-oss", arch="gpt-oss", n_layers=2, hidden=256, n_heads=8,
                           n_kv_heads=2, head_dim=64, ffn=128, vocab=1024, rope_theta=150000.0,
                           rope_neox=True, rope_scaling={"type": "yarn", "factor": 32.0,
                                                         "original_max_position_embeddings": 4096,
                                                         "beta_fast": 32.0, "beta_slow": 1.0},
                           attn_bias=True, attn_sinks=True, sliding_window=16, swa_every=2,
                           n_experts=8, n_experts_used=4, expert_ffn=128, swiglu_limit=7.0,
                           weight_qtype="BF16", embed_qtype="BF16", output_qtype="BF16",
                           expert_qtype="MXFP4")
    return ModelConfig(name="t-moe", arch="qwen3moe", n_layers=2, hidden=512, n_heads=8,
                       n_kv_heads=2, head_dim=64, ffn=256, vocab=1024, rms_eps=1e-6,
                       qk_norm=True, rope_neox=True, n_experts=16, n_experts_used=4,
                       expert_ffn=256, shared_expert_ffn=256, moe_softmax_after_topk=False,
                       weight_qtype="Q4_K", embed_qtype="F16", output_qtype="Q4_K",
                       expert_qtype="Q4_K")


@pytest.mark.parametrize("kind", ["gpt-oss", "moe-shared"])
def test_moe_model_matches_cpu_oracle(kind):
    """MoE families: prefill + decode logits vs the fp32 oracle.  A routing
    decision within rounding of a tie may flip between the two, so a few
    positions may drift; the bulk must match closely."""
    from swarmllm_b200.models.llama import LlamaCPU, LlamaGPU
    from swarmllm_b200.models.weights import RandomSource
    from swarmllm_b200.ops.attention import PagedKVCache
    cfg = _moe_cfg(kind)
    src = RandomSource(cfg, seed=11)
    gpu = LlamaGPU(cfg, src, DEV)
    cpu = LlamaCPU(cfg, src)
    ctx = gpu.make_context(64, 40, 256)
    kvg = PagedKVCache(cfg.n_layers, 8, cfg.n_kv_heads, cfg.head_dim, DEV)
    kvc = PagedKVCache(cfg.n_layers, 8, cfg.n_kv_heads, cfg.head_dim, "cpu", dtype=torch.float32)
    rng = np.random.default_rng(0)
    toks = rng.integers(0, cfg.vocab, 43)
    bt = np.tile(np.arange(8, dtype=np.int32), (64, 1))
    pos = np.arange(40)
    rows = list(range(40))
    lg = gpu.forward(_batch(toks[:40], pos, pos, bt[:40], DEV, rows), kvg, ctx)
    lc = cpu.forward(_batch(toks[:40], pos, pos, bt[:40], "cpu", rows), kvc)
    ctx.moe.check()
    cos = torch.nn.functional.cosine_similarity(lg.cpu().double(), lc.double(), dim=-1)
    assert float(cos.median()) > 0.999 and float((cos > 0.995).float().mean()) >= 0.9, cos
    for p in range(40, 43):
        lg = gpu.forward(_batch([toks[p]], [p], [p], bt[:1], DEV, [0]), kvg, ctx)
        lc = cpu.forward(_batch([toks[p]], [p], [p], bt[:1], "cpu", [0]), kvc)
        cos = torch.nn.functional.cosine_similarity(lg.cpu().double(), lc.double(), dim=-1)
        assert float(cos.min()) > 0.98, (p, cos)


def test_hybrid_model_matches_cpu_oracle():
    """Gated DeltaNet + gated attention (head_dim 256, partial RoPE) + MoE with
    a shared expert: two prefill chunks then decode steps, state carried."""
    import sys, os
    sys.path.insert(0, os.path.dirname(__file__))
    from test_hybrid_cpu import tiny_hybrid
    from swarmllm_b200.models.llama import LlamaCPU, LlamaGPU
    from swarmllm_b200.models.weights import RandomSource
    from swarmllm_b200.ops.attention import PagedKVCache
    cfg = tiny_hybrid()
    src = RandomSource(cfg, seed=5)
    gpu = LlamaGPU(cfg, src, DEV)
    cpu = LlamaCPU(cfg, src)
    ctx = gpu.make_context(128, 128, 256)
    spec = gpu.linear_state_spec()
    kvg = PagedKVCache(gpu.n_kv_layers, 16, cfg.n_kv_heads, cfg.head_dim, DEV)
    kvc = PagedKVCache(cpu.n_kv_layers, 16, cfg.n_kv_heads, cfg.head_dim, "cpu", dtype=torch.float32)
    kvg.add_linear_state(spec[0], 3, *spec[1:])
    kvc.add_linear_state(spec[0], 3, *spec[1:])
    rng = np.random.default_rng(1)
    toks = rng.integers(0, cfg.vocab, 200)
    bt = np.tile(np.arange(16, dtype=np.int32), (160, 1))

    def run(lo, hi):
        pos = np.arange(lo, hi)
        rows = list(range(hi - lo))
        outs = []
        for dev, model, kv in ((DEV, gpu, kvg), ("cpu", cpu, kvc)):
            b = _batch(toks[lo:hi], pos, pos, bt[:hi - lo], dev, rows)
            b.ssm_seqs = torch.tensor([[0, hi - lo, 1, lo]], dtype=torch.int32, device=dev)
            b.ssm_max_rows = hi - lo
            outs.append(model.forward(b, kv, ctx if dev == DEV else None))
        return torch.nn.functional.cosine_similarity(outs[0].cpu().double(), outs[1].double(), dim=-1)

    # recurrent (<= 32 rows) and chunked (> 32 rows, partial chunks) paths, state handed over
    for lo, hi in ((0, 24), (24, 40), (40, 41), (41, 141), (141, 142), (142, 143)):
        cos = run(lo, hi)
        assert float(cos.median()) > 0.999 and float(cos.min()) > 0.98, (lo, hi, cos)
    ctx.gemm.check()
    # the recurrent state itself
    st_g, st_c = kvg.ssm_state(0)[1].cpu(), kvc.ssm_state(0)[1]
    rel = float((st_g - st_c).norm() / st_c.norm())
    assert rel < 2e-2, rel


def test_hybrid_prefix_hit_gpu():
    """Hybrid model on the GPU engine: the recurrent state saved at the last
    page boundary before a prompt's end is restored for a repeat of the
    prompt, which then gives the same tokens with 48 prompt tokens skipped."""
    import sys, os
    sys.path.insert(0, os.path.dirname(__file__))
    from test_hybrid_cpu import tiny_hybrid
    from swarmllm_b200.engine import EngineConfig, LLMEngine, SamplingParams
    from swarmllm_b200.models.weights import RandomSource
    cfg = tiny_hybrid()
    ec = EngineConfig(max_model_len=128, max_running=4, max_step_tokens=64, prefill_chunk=64,
                      graph_sizes=(1, 2, 4))
    eng = LLMEngine.from_config(cfg, DEV, ec, source=RandomSource(cfg, seed=4))
    p = np.random.default_rng(3).integers(0, cfg.vocab, 53).tolist()
    sp = SamplingParams(max_tokens=6)
    o1 = eng.generate([p], sp)[0].token_ids
    assert eng.state_cache.saves == 1
    hits0 = eng.bm.prefix_hit_tokens
    o2 = eng.generate([p], sp)[0].token_ids
    assert eng.bm.prefix_hit_tokens - hits0 == 48 and eng.state_cache.restores == 1
    assert o1 == o2


def test_json_constraint_gpu_graph_path():
    """JSON-constrained decoding on the GPU engine, decode steps replayed from
    CUDA graphs (the constraint reads the graph's logits): the text is a valid
    JSON prefix, and the same for a sampled request."""
    from swarmllm_b200.engine import EngineConfig, LLMEngine, SamplingParams
    from swarmllm_b200.models.weights import RandomSource
    from swarmllm_b200.serve.json_guard import JsonConstraint, JsonPrefix
    from swarmllm_b200.serve.tokenizer import ByteTokenizer
    cfg = _cfg()
    tok = ByteTokenizer(cfg.vocab)
    eng = LLMEngine.from_config(cfg, DEV, EngineConfig(max_model_len=256, max_running=4,
                                                       max_step_tokens=128, prefill_chunk=64,
                                                       graph_sizes=(1, 2, 4)),
                                source=RandomSource(cfg, seed=5))
    prompt = tok.encode("json please")
    for temp in (0.0, 0.8):
        sp = SamplingParams(max_tokens=30, temperature=temp, seed=3, eos_token_id=tok.eos_id,
                            constraint=JsonConstraint(tok.token_str, tok.eos_id))
        outs = eng.generate([prompt, prompt], sp)
        for o in outs:
            text = tok.decode([t for t in o.token_ids if t != tok.eos_id])
            assert text.lstrip().startswith("{") and JsonPrefix().feed(text), text


def test_logit_bias_and_penalties_gpu_engine():
    """Logit adjustments on the GPU engine (eager sampling path, the
    apply_penalties kernel): a +100 bias pins greedy decoding to one token; a
    huge presence penalty never repeats a token."""
    from swarmllm_b200.engine import EngineConfig, LLMEngine, SamplingParams
    from swarmllm_b200.models.weights import RandomSource
    cfg = _cfg()
    eng = LLMEngine.from_config(cfg, DEV, EngineConfig(max_model_len=256, max_running=4,
                                                       max_step_tokens=128, prefill_chunk=64,
                                                       graph_sizes=(1, 2, 4)),
                                source=RandomSource(cfg, seed=5))
    prompt = np.random.default_rng(4).integers(0, cfg.vocab, 20).tolist()
    out = eng.generate([prompt], SamplingParams(max_tokens=6, logit_bias={42: 100.0}))[0].token_ids
    assert out == [42] * 6
    out = eng.generate([prompt], SamplingParams(max_tokens=30, presence_penalty=1e4))[0].token_ids
    assert len(set(out)) == len(out)
