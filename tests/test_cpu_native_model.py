"""The optimised CPU inference path (LlamaCPU(native=True): quantized weights
through the native int8-dot matmul, native paged attention and SwiGLU) against
the fp32 oracle (LlamaCPU(native=False)) on small random models of several
families: prefill logits, then a draft-tree decode step over the same cache."""
import numpy as np
import pytest
import torch

from test_families import family_cfg


def _run(m, cfg, T=40):
    from swarmllm_b200.models.llama import StepBatch
    from swarmllm_b200.ops.attention import PagedKVCache
    kv = PagedKVCache(cfg.n_layers, 8, cfg.n_kv_heads, cfg.head_dim, "cpu")
    toks = torch.from_numpy(np.random.default_rng(0).integers(0, cfg.vocab, T).astype(np.int32))
    pos = torch.arange(T, dtype=torch.int32)
    bt = torch.arange(8, dtype=torch.int32).repeat(T, 1)
    b = StepBatch(toks, pos, pos, bt, pos + 1, torch.arange(T), 128)
    pre = m.forward(b, kv)
    # a 3-node draft tree after the prompt: node 0 and 1 are siblings, node 2 a child of 1
    tt = torch.tensor([5, 6, 7], dtype=torch.int32)
    tp = torch.tensor([T, T, T + 1], dtype=torch.int32)
    slots = torch.tensor([T, T + 1, T + 2], dtype=torch.int32)
    masks = torch.tensor([0b001, 0b010, 0b110], dtype=torch.int64)
    b2 = StepBatch(tt, tp, slots, bt[:3], slots + 1, torch.arange(3), 128,
                   tree_mask=masks, tree_start=torch.full((3,), T, dtype=torch.int32))
    return pre, m.forward(b2, kv)


@pytest.mark.parametrize("fam,qtype", [("mistral", "Q4_K"), ("qwen3", "Q6_K"), ("phi3", "Q8_0"),
                                       ("gemma2", "Q4_K"), ("glm4", "Q8_0"), ("qwen2moe", "Q4_K"),
                                       ("qwen3moe", "Q8_0"), ("glm4moe", "Q4_K")])
def test_native_cpu_path_matches_oracle(fam, qtype):
    from swarmllm_b200.models.llama import LlamaCPU, _QWeight
    from swarmllm_b200.models.weights import RandomSource
    cfg = family_cfg(fam)
    cfg.weight_qtype = qtype
    cfg.output_qtype = qtype
    src = RandomSource(cfg, seed=3)
    ref, nat = LlamaCPU(cfg, src), LlamaCPU(cfg, src, native=True)
    assert isinstance(nat.layers[0].wo, _QWeight)
    if cfg.n_experts:
        moe = [L for L in nat.layers if L.moe]
        assert moe and isinstance(moe[0].eg, _QWeight) and moe[0].eg.expert_rows == cfg.expert_ffn
    assert isinstance(nat.head, _QWeight) != cfg.tie_embeddings   # a tied F16 head stays dense
    for r, n in zip(_run(ref, cfg), _run(nat, cfg)):
        rel = (n - r).norm() / r.norm()
        assert rel < 3e-2, rel
        cos = torch.nn.functional.cosine_similarity(n.flatten(), r.flatten(), dim=0)
        assert cos > 0.999


def test_native_delta_rule_matches_recurrence():
    from swarmllm_b200 import _native
    g_ = torch.Generator().manual_seed(0)
    T, nk, nv, D = 7, 2, 4, 32
    q = torch.nn.functional.normalize(torch.randn(T, nk, D, generator=g_), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(T, nk, D, generator=g_), dim=-1)
    v = torch.randn(T, nv, D, generator=g_)
    g = -torch.rand(T, nv, generator=g_)
    beta = torch.rand(T, nv, generator=g_)
    S0 = torch.randn(nv, D, D, generator=g_) * 0.1
    S = S0.clone()
    out = torch.from_numpy(_native.cpu_delta_rule(q.numpy(), k.numpy(), v.numpy(), g.numpy(),
                                                  beta.numpy(), S.numpy()))
    R = S0.clone()
    qq, kk = q.repeat_interleave(nv // nk, 1), k.repeat_interleave(nv // nk, 1)
    for t in range(T):
        R = R * torch.exp(g[t])[:, None, None]
        kv = torch.einsum("hij,hi->hj", R, kk[t])
        R = R + kk[t][:, :, None] * ((v[t] - kv) * beta[t][:, None])[:, None, :]
        assert torch.allclose(out[t], torch.einsum("hij,hi->hj", R, qq[t]), atol=1e-5)
    assert torch.allclose(S, R, atol=1e-5)


def test_native_hybrid_model_matches_oracle():
    from test_hybrid_cpu import tiny_hybrid
    from swarmllm_b200.models.llama import LlamaCPU, StepBatch
    from swarmllm_b200.models.weights import RandomSource
    from swarmllm_b200.ops.attention import PagedKVCache
    cfg = tiny_hybrid()
    src = RandomSource(cfg, seed=2)
    T = 20
    toks = torch.from_numpy(np.random.default_rng(0).integers(0, cfg.vocab, T).astype(np.int32))
    pos = torch.arange(T, dtype=torch.int32)
    bt = torch.arange(4, dtype=torch.int32).repeat(T, 1)
    outs = []
    for native in (False, True):
        m = LlamaCPU(cfg, src, native=native)
        kv = PagedKVCache(m.n_kv_layers, 4, cfg.n_kv_heads, cfg.head_dim, "cpu")
        spec = m.linear_state_spec()
        kv.add_linear_state(spec[0], 1, *spec[1:])
        res = []
        for lo, hi in ((0, 12), (12, T)):          # two chunks: the state carries over
            sl = slice(lo, hi)
            b = StepBatch(toks[sl], pos[sl], pos[sl], bt[sl], pos[sl] + 1,
                          torch.arange(hi - lo), 64,
                          ssm_seqs=torch.tensor([[0, hi - lo, 0, lo]], dtype=torch.int32))
            res.append(m.forward(b, kv))
        outs.append(torch.cat(res))
    rel = (outs[1] - outs[0]).norm() / outs[0].norm()
    assert rel < 3e-2, rel


def test_native_gpt_oss_mxfp4_experts():
    """gpt-oss: bf16 attention with sinks and a window (dequantized), MXFP4
    experts with biases and the clamped SwiGLU through the native matmul."""
    from swarmllm_b200.models.config import ModelConfig
    from swarmllm_b200.models.llama import LlamaCPU, _QWeight
    from swarmllm_b200.models.weights import RandomSource
    cfg = ModelConfig(name="t-oss", arch="gpt-oss", n_layers=2, hidden=256, n_heads=8,
                      n_kv_heads=2, head_dim=64, ffn=128, vocab=1024, rope_theta=150000.0,
                      rope_neox=True, attn_bias=True, attn_sinks=True, sliding_window=16,
                      swa_every=2, n_experts=8, n_experts_used=4, expert_ffn=128,
                      swiglu_limit=7.0, weight_qtype="BF16", embed_qtype="BF16",
                      output_qtype="BF16", expert_qtype="MXFP4")
    src = RandomSource(cfg, seed=4)
    ref, nat = LlamaCPU(cfg, src), LlamaCPU(cfg, src, native=True)
    assert isinstance(nat.layers[0].eg, _QWeight) and isinstance(nat.layers[0].ed, _QWeight)
    for r, n in zip(_run(ref, cfg), _run(nat, cfg)):
        rel = (n - r).norm() / r.norm()
        assert rel < 3e-2, rel
