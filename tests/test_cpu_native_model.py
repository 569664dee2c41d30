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
                                       ("gemma2", "Q4_K"), ("glm4", "Q8_0")])
def test_native_cpu_path_matches_oracle(fam, qtype):
    from swarmllm_b200.models.llama import LlamaCPU, _QWeight
    from swarmllm_b200.models.weights import RandomSource
    cfg = family_cfg(fam)
    cfg.weight_qtype = qtype
    cfg.output_qtype = qtype
    src = RandomSource(cfg, seed=3)
    ref, nat = LlamaCPU(cfg, src), LlamaCPU(cfg, src, native=True)
    assert isinstance(nat.layers[0].wo, _QWeight)
    assert isinstance(nat.head, _QWeight) != cfg.tie_embeddings   # a tied F16 head stays dense
    for r, n in zip(_run(ref, cfg), _run(nat, cfg)):
        rel = (n - r).norm() / r.norm()
        assert rel < 3e-2, rel
        cos = torch.nn.functional.cosine_similarity(n.flatten(), r.flatten(), dim=0)
        assert cos > 0.999
