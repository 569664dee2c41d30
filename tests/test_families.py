"""Model families beyond Llama (CPU): GGUF metadata of each family maps to
the family's options, a random-init GGUF of each family round-trips through
the file, and the CPU model runs it (the GPU kernels are checked against this
CPU model in tests/test_families_gpu.py)."""
import numpy as np
import pytest
import torch


def family_cfg(fam: str):
    """A small model of each family (head_dim 96 for phi3, as Phi-3-mini)."""
    from swarmllm_b200.models.config import ModelConfig, apply_family
    kw = dict(name=f"tiny-{fam}", arch=fam, n_layers=3, hidden=512, n_heads=8, n_kv_heads=2,
              head_dim=64, ffn=1024, vocab=1024, weight_qtype="Q8_0", embed_qtype="F16",
              output_qtype="Q8_0", rope_theta=10000.0, sliding_window=24)
    if fam == "phi3":
        kw.update(hidden=768, n_heads=8, n_kv_heads=8, head_dim=96, ffn=1536)
    if fam in ("qwen2moe", "qwen3moe", "glm4moe"):
        kw.update(n_experts=8, n_experts_used=2, expert_ffn=256, weight_qtype="Q4_K",
                  output_qtype="Q4_K", shared_expert_ffn=256 if fam != "qwen3moe" else 0)
    if fam == "glm4moe":
        kw.update(moe_dense_layers=1, moe_scale=1.5, qk_norm=True)
    cfg = apply_family(ModelConfig(**kw))
    if fam == "gemma3":
        cfg.rope_theta = 1e6
    return cfg


FAMILIES = ["mistral", "qwen2", "qwen3", "qwen2moe", "qwen3moe", "gemma", "gemma2", "gemma3",
            "phi3", "glm4", "glm4moe"]


def test_family_options():
    from swarmllm_b200.models.config import ModelConfig, from_gguf_metadata
    base = {"block_count": 2, "embedding_length": 512, "attention.head_count": 8,
            "attention.head_count_kv": 2, "feed_forward_length": 1024, "vocab_size": 1000,
            "context_length": 4096}

    def md(arch, **extra):
        d = {"general.architecture": arch}
        d.update({f"{arch}.{k}": v for k, v in {**base, **extra}.items()})
        return d
    c = from_gguf_metadata(md("qwen2"))
    assert c.attn_bias and not c.has_out_bias and c.rope_neox
    c = from_gguf_metadata(md("qwen3"))
    assert c.qk_norm and c.rope_neox and not c.attn_bias
    c = from_gguf_metadata(md("gemma2", attn_logit_softcapping=50.0, final_logit_softcapping=30.0))
    assert c.act == "gelu" and c.post_norms and c.attn_softcap == 50.0 and c.final_softcap == 30.0
    assert abs(c.embed_scale - 512 ** 0.5) < 1e-9 and c.tie_embeddings
    c = from_gguf_metadata(md("gemma3", **{"attention.sliding_window": 1024}))
    assert c.qk_norm and c.swa_pattern == 6 and c.rope_local_theta == 10000.0
    assert [c.is_swa(i) for i in range(7)] == [True] * 5 + [False, True]
    c = from_gguf_metadata(md("phi3"))
    assert c.fused_qkv and c.fused_gate_up
    c = from_gguf_metadata(md("glm4", **{"attention.key_length": 128}))
    assert c.fused_qkv and c.post_norms and c.rot_dim == 64 and c.attn_bias
    c = from_gguf_metadata(md("qwen2moe", expert_count=8, expert_used_count=2))
    assert not c.moe_softmax_after_topk
    with pytest.raises(ValueError):
        from_gguf_metadata(md("starcoder2"))


@pytest.mark.parametrize("fam", FAMILIES)
def test_family_gguf_roundtrip_and_cpu_forward(fam, tmp_path):
    from swarmllm_b200.models.llama import LlamaCPU, StepBatch
    from swarmllm_b200.models.weights import GgufSource, RandomSource, write_random_gguf
    from swarmllm_b200.ops.attention import PagedKVCache
    cfg = family_cfg(fam)
    path = write_random_gguf(cfg, str(tmp_path / f"{fam}.gguf"), seed=2)
    src = GgufSource(path)
    assert src.cfg.arch == fam and src.cfg.fused_qkv == cfg.fused_qkv
    m1, m2 = LlamaCPU(src.cfg, src), LlamaCPU(cfg, RandomSource(cfg, seed=2))
    T = 30
    toks = torch.from_numpy(np.random.default_rng(0).integers(0, cfg.vocab, T).astype(np.int32))
    pos = torch.arange(T, dtype=torch.int32)
    bt = torch.arange(4, dtype=torch.int32).repeat(T, 1)
    outs = []
    for m in (m1, m2):
        kv = PagedKVCache(cfg.n_layers, 4, cfg.n_kv_heads, cfg.head_dim, "cpu", dtype=torch.float32)
        b = StepBatch(toks, pos, pos, bt, pos + 1, torch.tensor([T - 1]), 64)
        outs.append(m.forward(b, kv))
    assert torch.isfinite(outs[0]).all()
    assert torch.allclose(outs[0], outs[1])


def test_glm4moe_file_layout_and_metadata(tmp_path):
    """GLM-4.5 files: the FFN pre-norm is named post_attention_norm, the first
    layers are dense, routed layers carry the selection bias and an ungated
    shared expert; the file's own keys (no engine blob) give the routing."""
    from swarmllm_b200.gguf.file import GGUFReader
    from swarmllm_b200.models.config import from_gguf_metadata, to_gguf_metadata
    from swarmllm_b200.models.weights import GgufSource, RandomSource, write_random_gguf
    cfg = family_cfg("glm4moe")
    path = write_random_gguf(cfg, str(tmp_path / "g.gguf"), seed=1)
    names = set(GGUFReader(path).tensors)
    assert "blk.0.post_attention_norm.weight" in names and "blk.0.ffn_norm.weight" not in names
    assert "blk.0.ffn_gate.weight" in names and "blk.0.ffn_gate_exps.weight" not in names
    assert "blk.1.ffn_gate_exps.weight" in names and "blk.1.exp_probs_b.bias" in names
    assert "blk.1.ffn_gate_inp_shexp.weight" not in names
    src = GgufSource(path)
    a, _, _ = src.get("blk.1.ffn_norm.weight")
    b, _, _ = RandomSource(cfg, seed=1).get("blk.1.ffn_norm.weight")
    assert torch.equal(a, b)
    md = to_gguf_metadata(cfg)
    md.pop("swarmllm.config")
    md["general.architecture"] = "glm4moe"
    md["glm4moe.block_count"] = cfg.n_layers + 1
    md["glm4moe.nextn_predict_layers"] = 1
    c = from_gguf_metadata(md)
    assert c.n_layers == cfg.n_layers and c.moe_gating == "sigmoid" and c.moe_mode == 2
    assert c.moe_dense_layers == 1 and c.moe_scale == 1.5 and c.moe_norm_topk
    assert c.shared_expert_ffn == cfg.expert_ffn and not c.shared_expert_gated
    assert [c.is_moe_layer(i) for i in range(3)] == [False, True, True]


def test_sigmoid_routing_oracle():
    """Sigmoid gating: the selection bias decides which experts run, the
    weights are the unbiased scores (renormalised, scaled)."""
    from swarmllm_b200.models.llama import LlamaCPU, _GpuLayer
    cfg = family_cfg("glm4moe")
    m = LlamaCPU.__new__(LlamaCPU)
    m.cfg = cfg
    L = _GpuLayer()
    E, H, F = cfg.n_experts, cfg.hidden, cfg.expert_ffn
    g = torch.Generator().manual_seed(0)
    L.wr = torch.randn(E, H, generator=g) * 0.05
    L.br = None
    L.sel_b = torch.zeros(E)
    L.sel_b[5] = 10.0                               # expert 5 always selected
    L.eg = torch.randn(E, F, H, generator=g) * 0.02
    L.eu = torch.randn(E, F, H, generator=g) * 0.02
    L.ed = torch.randn(E, H, F, generator=g) * 0.02
    L.ebg = L.ebu = L.ebd = None
    L.sg = L.sgi = None
    x = torch.randn(3, H, generator=g)
    y = m._moe(x, L)
    score = torch.sigmoid(x @ L.wr.T)
    want = torch.zeros_like(x)
    for t in range(3):
        sel = torch.topk(score[t] + L.sel_b, 2).indices
        assert 5 in sel.tolist()
        w = score[t, sel] / score[t, sel].sum() * cfg.moe_scale
        for e, we in zip(sel.tolist(), w):
            a = torch.nn.functional.silu(x[t] @ L.eg[e].T) * (x[t] @ L.eu[e].T)
            want[t] += we * (a @ L.ed[e].T)
    assert torch.allclose(y, want, atol=1e-5)
