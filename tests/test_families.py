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
    if fam == "llama4":  # layers 1 and 3 routed, layer 3 without RoPE
        kw.update(n_layers=4, n_experts=8, n_experts_used=1, expert_ffn=256,
                  shared_expert_ffn=256, moe_every=2, weight_qtype="Q4_K", output_qtype="Q4_K",
                  sliding_window=0)
    if fam == "granite":
        kw.update(embed_scale=12.0, residual_scale=0.22, logit_scale=8.0, attn_scale=0.0078125)
    cfg = apply_family(ModelConfig(**kw))
    if fam == "gemma3":
        cfg.rope_theta = 1e6
    return cfg


FAMILIES = ["mistral", "qwen2", "qwen3", "qwen2moe", "qwen3moe", "gemma", "gemma2", "gemma3",
            "phi3", "glm4", "glm4moe", "llama4", "granite"]


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
    c = from_gguf_metadata({**md("gemma2"), "gemma2.block_count": 46, "gemma2.embedding_length": 4608,
                            "gemma2.attention.head_count": 32, "gemma2.attention.key_length": 128})
    assert abs(c.softmax_scale - 144 ** -0.5) < 1e-12          # Gemma 2 27B
    c = from_gguf_metadata({**md("gemma3"), "gemma3.attention.key_length": 128})
    assert abs(c.softmax_scale - 128 ** -0.5) < 1e-12          # other sizes: head width
    c = from_gguf_metadata(md("phi3"))
    assert c.fused_qkv and c.fused_gate_up
    c = from_gguf_metadata(md("glm4", **{"attention.key_length": 128}))
    assert c.fused_qkv and c.post_norms and c.rot_dim == 64 and c.attn_bias
    c = from_gguf_metadata(md("qwen2moe", expert_count=8, expert_used_count=2))
    assert not c.moe_softmax_after_topk
    c = from_gguf_metadata(md("llama4", expert_count=16, expert_used_count=1,
                              expert_feed_forward_length=256, interleave_moe_layer_step=2))
    assert c.nope_every == 4 and c.qk_rms_plain and not c.rope_neox
    assert c.moe_gating == "sigmoid" and c.moe_weight_input and not c.moe_norm_topk
    assert not c.moe_sel_bias and not c.shared_expert_gated and c.shared_expert_ffn == 256
    assert [c.is_moe_layer(i) for i in range(4)] == [False, True, False, True]
    assert [c.is_nope(i) for i in range(8)] == [False, False, False, True] * 2
    c = from_gguf_metadata(md("llama4", expert_count=128, expert_used_count=1))
    assert not c.qk_rms_plain and all(c.is_moe_layer(i) for i in range(2))  # Maverick-style
    c = from_gguf_metadata(md("granite", embedding_scale=12.0, residual_scale=0.22,
                              logit_scale=8.0, **{"attention.scale": 0.0078125}))
    assert (c.embed_scale, c.residual_scale, c.logit_scale, c.attn_scale) == (12.0, 0.22, 8.0, 0.0078125)
    c = from_gguf_metadata(md("granite", embedding_scale=1.0, residual_scale=1.0, logit_scale=1.0))
    assert not c.embed_scale and not c.residual_scale and not c.logit_scale
    c = from_gguf_metadata(md("qwen3vl", **{"attention.key_length": 128}))
    assert c.arch == "qwen3" and c.qk_norm and c.head_dim == 128
    assert from_gguf_metadata(md("qwen2vl")).attn_bias
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


def _plain_forward(cfg, src, tokens):
    """A dense decoder written out step by step (fp32, no cache) for the
    llama4 and granite options: NoPE layers, per-head q/k RMS without a
    weight applied after interleaved RoPE, the embedding / residual /
    attention / logit multipliers."""
    from swarmllm_b200.models.llama import _f32
    from swarmllm_b200.models.config import rope_inv_freq

    def w(name):
        t, qt, shape = src.get(name)
        return _f32(t, qt, shape)

    def rms(x, g=1.0):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + cfg.rms_eps) * g

    T, d = len(tokens), cfg.head_dim
    inv, af = rope_inv_freq(cfg)
    ang = torch.arange(T, dtype=torch.float32)[:, None] * torch.from_numpy(inv)[None, :]
    cos, sin = (torch.cos(ang) * af)[:, None, :], (torch.sin(ang) * af)[:, None, :]

    def rope(x):  # GGML "norm": pairs (2i, 2i+1)
        a, b = x[..., 0::2], x[..., 1::2]
        out = torch.empty_like(x)
        out[..., 0::2], out[..., 1::2] = a * cos - b * sin, b * cos + a * sin
        return out

    h = w("token_embd.weight")[torch.as_tensor(tokens).long()]
    if cfg.embed_scale:
        h = h * cfg.embed_scale
    rs = cfg.residual_scale or 1.0
    mask = torch.full((T, T), float("-inf")).triu(1)
    for i in range(cfg.n_layers):
        b = f"blk.{i}."
        x = rms(h, w(b + "attn_norm.weight"))
        q = (x @ w(b + "attn_q.weight").T).view(T, cfg.n_heads, d)
        k = (x @ w(b + "attn_k.weight").T).view(T, cfg.n_kv_heads, d)
        v = (x @ w(b + "attn_v.weight").T).view(T, cfg.n_kv_heads, d)
        if (i + 1) % 4 != 0 or not cfg.nope_every:
            q, k = rope(q), rope(k)
            if cfg.qk_rms_plain:
                q, k = rms(q), rms(k)
        rep = cfg.n_heads // cfg.n_kv_heads
        k, v = k.repeat_interleave(rep, 1), v.repeat_interleave(rep, 1)
        s = torch.einsum("qhd,khd->hqk", q, k) * cfg.softmax_scale + mask
        a = torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), v).reshape(T, -1)
        h = h + (a @ w(b + "attn_output.weight").T) * rs
        x = rms(h, w(b + "ffn_norm.weight"))
        g, u = x @ w(b + "ffn_gate.weight").T, x @ w(b + "ffn_up.weight").T
        h = h + ((torch.nn.functional.silu(g) * u) @ w(b + "ffn_down.weight").T) * rs
    logits = rms(h, w("output_norm.weight")) @ w("output.weight").T
    return logits / (cfg.logit_scale or 1.0)


@pytest.mark.parametrize("fam", ["llama4", "granite"])
def test_llama4_granite_match_plain_forward(fam):
    """The CPU model's llama4 (dense layers: NoPE every 4th layer, plain q/k
    RMS after RoPE) and granite (four multipliers) equal a forward written
    out step by step from the same weights."""
    from swarmllm_b200.models.llama import LlamaCPU, StepBatch
    from swarmllm_b200.models.weights import RandomSource
    from swarmllm_b200.ops.attention import PagedKVCache
    cfg = family_cfg(fam)
    cfg.n_experts = cfg.moe_every = 0   # dense layers here; routed ones: test below
    cfg.weight_qtype = cfg.output_qtype = "Q8_0"
    src = RandomSource(cfg, seed=5, std=0.05)
    m = LlamaCPU(cfg, src)
    T = 12
    toks = np.random.default_rng(1).integers(0, cfg.vocab, T).astype(np.int32)
    pos = torch.arange(T, dtype=torch.int32)
    bt = torch.arange(4, dtype=torch.int32).repeat(T, 1)
    kv = PagedKVCache(cfg.n_layers, 4, cfg.n_kv_heads, cfg.head_dim, "cpu", dtype=torch.float32)
    b = StepBatch(torch.from_numpy(toks), pos, pos, bt, pos + 1, torch.arange(T), 64)
    got = m.forward(b, kv)
    want = _plain_forward(cfg, src, toks.tolist())
    assert torch.allclose(got, want, rtol=1e-4, atol=1e-4), (got - want).abs().max()
    if fam == "llama4":  # the options matter: without NoPE the result differs
        cfg2 = family_cfg(fam)
        cfg2.n_experts = cfg2.moe_every = cfg2.nope_every = 0
        cfg2.weight_qtype = cfg2.output_qtype = "Q8_0"
        other = LlamaCPU(cfg2, RandomSource(cfg2, seed=5, std=0.05)).forward(
            b, PagedKVCache(cfg.n_layers, 4, cfg.n_kv_heads, cfg.head_dim, "cpu",
                            dtype=torch.float32))
        assert not torch.allclose(other, want, rtol=1e-3, atol=1e-3)


def test_llama4_routing_weights_the_expert_input():
    """llama4 experts: sigmoid scores, no renormalisation, and the chosen
    expert computes down(silu(gate(w x)) * up(w x)), not w * expert(x);
    the shared expert is ungated."""
    from swarmllm_b200.models.llama import LlamaCPU, _GpuLayer
    cfg = family_cfg("llama4")
    m = LlamaCPU.__new__(LlamaCPU)
    m.cfg, m.native = cfg, False
    L = _GpuLayer()
    E, H, F = cfg.n_experts, cfg.hidden, cfg.expert_ffn
    g = torch.Generator().manual_seed(0)
    L.wr = torch.randn(E, H, generator=g) * 0.05
    L.br = L.sel_b = None
    L.eg, L.eu, L.ed = (torch.randn(E, F, H, generator=g) * 0.05,
                        torch.randn(E, F, H, generator=g) * 0.05,
                        torch.randn(E, H, F, generator=g) * 0.05)
    L.ebg = L.ebu = L.ebd = None
    L.sg, L.su, L.sd = (torch.randn(F, H, generator=g) * 0.05, torch.randn(F, H, generator=g) * 0.05,
                        torch.randn(H, F, generator=g) * 0.05)
    L.sgi = None
    x = torch.randn(4, H, generator=g)
    y = m._moe(x, L)
    silu = torch.nn.functional.silu
    want = torch.zeros_like(x)
    for t in range(4):
        score = torch.sigmoid(x[t] @ L.wr.T)
        e = int(torch.argmax(score))
        xi = score[e] * x[t]
        want[t] = (silu(xi @ L.eg[e].T) * (xi @ L.eu[e].T)) @ L.ed[e].T
        want[t] += (silu(x[t] @ L.sg.T) * (x[t] @ L.su.T)) @ L.sd.T
    assert torch.allclose(y, want, atol=1e-5)


def test_gpu_model_refuses_unbuilt_options():
    """The GPU model names what its kernels lack instead of running it wrong."""
    from swarmllm_b200.models.llama import LlamaGPU
    for fam in ("llama4", "granite"):
        with pytest.raises(NotImplementedError, match=fam):
            LlamaGPU(family_cfg(fam), None, "cpu")


def test_rope_freqs_tensor_scales_llama_rope(tmp_path):
    """A Llama 3.x file's rope_freqs tensor (per-pair divisors, how llama3
    scaling is stored) divides the rotary frequencies of the loaded model."""
    from swarmllm_b200.gguf import quants as Q
    from swarmllm_b200.gguf.file import GGUFWriter
    from swarmllm_b200.models.config import rope_inv_freq, tiny_llama, to_gguf_metadata
    from swarmllm_b200.models.layout import file_specs, to_file
    from swarmllm_b200.models.weights import GgufSource, RandomSource, tensor_specs
    cfg = tiny_llama()
    src = RandomSource(cfg, seed=0)
    w = GGUFWriter(cfg.arch)
    md = to_gguf_metadata(cfg)
    md.pop("swarmllm.config")
    for k, v in md.items():
        w.add(k, v)
    for name, shape, qt in file_specs(cfg, tensor_specs(cfg)):
        w.add_tensor(name, to_file(cfg, name, shape, qt, lambda n: src.get(n)[0].numpy()), qt, shape)
    half = cfg.rot_dim // 2
    factors = np.where(np.arange(half) < half // 2, 1.0, 8.0).astype(np.float32)
    w.add_tensor("rope_freqs.weight", factors, Q.F32, (half,))
    path = str(tmp_path / "l3.gguf")
    w.write(path)
    got = GgufSource(path).cfg
    assert got.rope_factors == factors.tolist()
    inv, _ = rope_inv_freq(got)
    plain, _ = rope_inv_freq(cfg)
    assert np.allclose(inv, plain / factors)
