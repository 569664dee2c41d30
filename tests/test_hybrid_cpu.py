"""Hybrid (gated DeltaNet + gated attention + MoE) model on the CPU engine:
the recurrent state carried across prefill chunks and decode steps."""
import numpy as np
import pytest
import torch


def tiny_hybrid():
    from swarmllm_b200.models.config import ModelConfig
    return ModelConfig(name="t-hybrid", arch="qwen3next", n_layers=4, hidden=256, n_heads=4,
                       n_kv_heads=2, head_dim=256, ffn=256, vocab=512, rope_theta=1e7,
                       rope_neox=True, rope_dim=64, rms_eps=1e-6, qk_norm=True,
                       attn_output_gate=True, n_experts=8, n_experts_used=2, expert_ffn=256,
                       shared_expert_ffn=256, moe_softmax_after_topk=False,
                       full_attn_interval=4, ssm_k_heads=2, ssm_v_heads=4, ssm_head_dim=128,
                       ssm_conv_kernel=4, weight_qtype="Q4_K", embed_qtype="F16",
                       output_qtype="Q4_K", expert_qtype="Q4_K")


def test_hybrid_layout():
    cfg = tiny_hybrid()
    assert [cfg.is_linear_attn(i) for i in range(4)] == [True, True, True, False]


def test_hybrid_chunked_prefill_matches_single_chunk():
    from swarmllm_b200.engine import EngineConfig, LLMEngine, SamplingParams
    from swarmllm_b200.models.weights import RandomSource
    cfg = tiny_hybrid()
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, cfg.vocab, n).tolist() for n in (13, 30)]
    outs = []
    for chunk in (64, 8):
        ec = EngineConfig(max_model_len=96, max_running=4, max_step_tokens=64, prefill_chunk=chunk)
        eng = LLMEngine.from_config(cfg, "cpu", ec, source=RandomSource(cfg, seed=4))
        outs.append([o.token_ids for o in eng.generate(prompts, SamplingParams(max_tokens=6))])
    assert outs[0] == outs[1]


def _hyb_engine(entries):
    from swarmllm_b200.engine import EngineConfig, LLMEngine
    from swarmllm_b200.models.weights import RandomSource
    cfg = tiny_hybrid()
    ec = EngineConfig(max_model_len=128, max_running=4, max_step_tokens=64, prefill_chunk=64,
                      state_cache_entries=entries)
    return LLMEngine.from_config(cfg, "cpu", ec, source=RandomSource(cfg, seed=4))


def test_hybrid_prefix_hit_restores_recurrent_state():
    """The state saved at the last page boundary before a prompt's end lets a
    later prompt with that prefix skip it: same output as without any cache."""
    from swarmllm_b200.engine import SamplingParams
    sp = SamplingParams(max_tokens=5)
    rng = np.random.default_rng(3)
    base = rng.integers(0, 512, 50).tolist()
    p1 = base + [7, 8, 9]                               # 53 tokens: state saved at 48
    p2 = base[:48] + rng.integers(0, 512, 20).tolist()  # shares 3 full pages
    eng = _hyb_engine(8)
    assert eng.ecfg.prefix_cache and eng.state_cache is not None
    o1 = eng.generate([p1], sp)[0].token_ids
    assert eng.state_cache.saves == 1
    hits0 = eng.bm.prefix_hit_tokens
    o2 = eng.generate([p2], sp)[0].token_ids
    assert eng.bm.prefix_hit_tokens - hits0 == 48 and eng.state_cache.restores == 1
    o1b = eng.generate([p1], sp)[0].token_ids           # the first prompt again: hit at 48
    assert eng.state_cache.restores == 2
    ref = _hyb_engine(0)
    assert not ref.ecfg.prefix_cache
    assert o1 == o1b == ref.generate([p1], sp)[0].token_ids
    assert o2 == ref.generate([p2], sp)[0].token_ids


def test_hybrid_hit_needs_saved_state():
    """KV pages alone give no hit: with the saved state evicted the prompt is
    recomputed from the start."""
    from swarmllm_b200.engine import SamplingParams
    sp = SamplingParams(max_tokens=3)
    rng = np.random.default_rng(4)
    a = rng.integers(0, 512, 40).tolist()
    b = rng.integers(0, 512, 40).tolist()
    eng = _hyb_engine(1)                                # one entry: b's save evicts a's
    eng.generate([a], sp)
    eng.generate([b], sp)
    hits0 = eng.bm.prefix_hit_tokens
    out = eng.generate([a], sp)[0].token_ids
    assert eng.bm.prefix_hit_tokens == hits0
    assert out == _hyb_engine(0).generate([a], sp)[0].token_ids
