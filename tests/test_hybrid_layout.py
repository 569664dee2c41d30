"""Hybrid families' file order vs the kernels' order (models/layout.py):
Qwen3-Next files interleave beta and alpha per key head; Qwen 3.5 files tile
the value heads over the key heads and keep beta and alpha apart.  A random
GGUF written in the file order and read back gives the kernels' tensors, and
the CPU model on it matches the one on the kernel-order source."""
import dataclasses

import numpy as np
import pytest
import torch

from test_hybrid_cpu import tiny_hybrid


def test_head_permutations():
    from swarmllm_b200.models import layout as Lo
    # Qwen 3.5: file head f reads key head f % nk; kernel head g reads key head g // r
    nk, nv = 2, 6
    p = Lo.head_perm("qwen35", nk, nv)
    assert sorted(p.tolist()) == list(range(nv))
    r = nv // nk
    for g in range(nv):
        assert p[g] % nk == g // r
    assert Lo.head_perm("qwen3next", nk, nv).tolist() == list(range(nv))
    # Qwen3-Next ssm_ba: per key head r betas then r alphas
    assert Lo.ba_rows(2, 4).tolist() == [0, 1, 4, 5, 2, 3, 6, 7]


def _cfg(arch, qtype, moe):
    cfg = dataclasses.replace(tiny_hybrid(), arch=arch, weight_qtype=qtype, output_qtype=qtype,
                              expert_qtype=qtype)
    if not moe:
        cfg = dataclasses.replace(cfg, n_experts=0, n_experts_used=0, expert_ffn=0,
                                  shared_expert_ffn=0)
    return cfg


@pytest.mark.parametrize("arch,qtype,moe", [("qwen3next", "Q4_K", True), ("qwen35", "Q8_0", False),
                                            ("qwen35moe", "Q8_0", True), ("qwen35", "Q4_K", False)])
def test_file_order_roundtrip(arch, qtype, moe, tmp_path):
    from swarmllm_b200.gguf.file import GGUFReader
    from swarmllm_b200.models.llama import LlamaCPU, StepBatch
    from swarmllm_b200.models.weights import GgufSource, RandomSource, write_random_gguf
    from swarmllm_b200.ops.attention import PagedKVCache
    cfg = _cfg(arch, qtype, moe)
    path = write_random_gguf(cfg, str(tmp_path / f"{arch}.gguf"), seed=5)
    names = set(GGUFReader(path).tensors)
    if arch == "qwen3next":
        assert "blk.0.ssm_ba.weight" in names
    else:
        assert "blk.0.ssm_beta.weight" in names and "blk.0.ssm_alpha.weight" in names
        assert "blk.0.ssm_ba.weight" not in names
    fsrc, rsrc = GgufSource(path), RandomSource(cfg, seed=5)
    exact = not (arch == "qwen35" and qtype == "Q4_K")   # Q4_K blocks span two 128-wide heads
    for n in ("blk.0.attn_qkv.weight", "blk.0.attn_gate.weight", "blk.0.ssm_ba.weight",
              "blk.0.ssm_conv1d.weight", "blk.0.ssm_dt.bias", "blk.0.ssm_a",
              "blk.0.ssm_out.weight"):
        a, qa, sa = fsrc.get(n)
        b, qb, sb = rsrc.get(n)
        assert tuple(sa) == tuple(sb), n
        if exact or n != "blk.0.ssm_out.weight":
            assert qa == qb and torch.equal(a, b), n
    if not exact:   # ssm_out came back as F16 columns in the kernels' order
        from swarmllm_b200.gguf import quants as Q
        a, qa, sa = fsrc.get("blk.0.ssm_out.weight")
        b, qb, sb = rsrc.get("blk.0.ssm_out.weight")
        assert qa == Q.F16
        fa = Q.dequantize(a.numpy(), qa).reshape(sa)
        fb = Q.dequantize(b.numpy(), qb).reshape(sb)
        assert np.abs(fa - fb).max() < 0.02 * np.abs(fb).max()
    T = 12
    toks = torch.from_numpy(np.random.default_rng(1).integers(0, cfg.vocab, T).astype(np.int32))
    pos = torch.arange(T, dtype=torch.int32)
    bt = torch.arange(4, dtype=torch.int32).repeat(T, 1)
    outs = []
    for src in (fsrc, rsrc):
        m = LlamaCPU(fsrc.cfg if src is fsrc else cfg, src)
        kv = PagedKVCache(m.n_kv_layers, 4, cfg.n_kv_heads, cfg.head_dim, "cpu", dtype=torch.float32)
        kv.add_linear_state(*m.linear_state_spec()[:1], 1, *m.linear_state_spec()[1:])
        b = StepBatch(toks, pos, pos, bt, pos + 1, torch.tensor([T - 1]), 64,
                      ssm_seqs=torch.tensor([[0, T, 0, 0]], dtype=torch.int32))
        outs.append(m.forward(b, kv))
    if exact:
        assert torch.allclose(outs[0], outs[1], atol=1e-5)
    else:
        assert torch.nn.functional.cosine_similarity(outs[0].flatten(), outs[1].flatten(), 0) > 0.99


def test_qwen35_metadata_without_engine_keys():
    """A Qwen 3.5 file's own keys (no engine config blob) give the geometry."""
    from swarmllm_b200.models.config import from_gguf_metadata, to_gguf_metadata
    cfg = _cfg("qwen35", "Q4_K", False)
    md = to_gguf_metadata(cfg)
    md.pop("swarmllm.config")
    md["general.architecture"] = "qwen35"
    c = from_gguf_metadata(md)
    assert (c.ssm_k_heads, c.ssm_v_heads, c.ssm_head_dim, c.full_attn_interval) == (2, 4, 128, 4)
    assert c.attn_output_gate and c.qk_norm and c.rope_neox and not c.n_experts


@pytest.mark.parametrize("arch", ["qwen35", "gpt-oss"])
def test_ffn_pre_norm_file_name(arch, tmp_path):
    """gpt-oss, GLM-4.5 and the Qwen hybrids' files name the norm before the
    feed-forward post_attention_norm; the engine reads it as ffn_norm."""
    from swarmllm_b200.gguf.file import GGUFReader
    from swarmllm_b200.models.config import ModelConfig
    from swarmllm_b200.models.weights import GgufSource, RandomSource, write_random_gguf
    if arch == "gpt-oss":
        cfg = ModelConfig(name="t-oss", arch="gpt-oss", n_layers=2, hidden=256, n_heads=8,
                          n_kv_heads=2, head_dim=64, ffn=128, vocab=512, attn_bias=True,
                          attn_sinks=True, sliding_window=16, swa_every=2, n_experts=4,
                          n_experts_used=2, expert_ffn=128, swiglu_limit=7.0,
                          weight_qtype="Q8_0", embed_qtype="Q8_0", output_qtype="Q8_0",
                          expert_qtype="MXFP4")
    else:
        cfg = _cfg("qwen35", "Q8_0", False)
    path = write_random_gguf(cfg, str(tmp_path / "m.gguf"), seed=2)
    names = set(GGUFReader(path).tensors)
    assert "blk.0.post_attention_norm.weight" in names and "blk.0.ffn_norm.weight" not in names
    a, _, _ = GgufSource(path).get("blk.1.ffn_norm.weight")
    b, _, _ = RandomSource(cfg, seed=2).get("blk.1.ffn_norm.weight")
    assert torch.equal(a, b)
