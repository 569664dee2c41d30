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
        assert eng.ecfg.prefix_cache is False
        outs.append([o.token_ids for o in eng.generate(prompts, SamplingParams(max_tokens=6))])
    assert outs[0] == outs[1]
