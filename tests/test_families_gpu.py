"""Every model family's GPU forward (sm_100a kernels: fused epilogues incl. the
GELU gate and the post-norm residual epilogue, soft-capped / head_dim-96
attention, per-layer RoPE bases) against its CPU fp32 oracle: prefill of one
sequence, then decode steps; logits cosine > 0.999."""
import numpy as np
import pytest
import torch

from test_families import FAMILIES, family_cfg

# llama4 and granite's residual multiplier run on the CPU model only (the GPU
# model refuses them by name: test_gpu_model_refuses_unbuilt_options)
GPU_FAMILIES = [f for f in FAMILIES if f not in ("llama4", "granite")]

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _batch(tokens, positions, bt, device, sample_rows):
    from swarmllm_b200.models.llama import StepBatch
    t = lambda a, dt=torch.int32: torch.as_tensor(np.asarray(a), dtype=dt, device=device)
    return StepBatch(t(tokens), t(positions), t(positions), t(bt), t(np.asarray(positions) + 1),
                     t(sample_rows, torch.int64), 256)


@pytest.mark.parametrize("fam", GPU_FAMILIES)
def test_family_gpu_matches_cpu_oracle(fam):
    from swarmllm_b200.models.llama import LlamaCPU, LlamaGPU
    from swarmllm_b200.models.weights import RandomSource
    from swarmllm_b200.ops.attention import PagedKVCache
    cfg = family_cfg(fam)
    src = RandomSource(cfg, seed=3)
    gpu, cpu = LlamaGPU(cfg, src, DEV), LlamaCPU(cfg, src)
    ctx = gpu.make_context(64, 8, 256)
    kvg = PagedKVCache(cfg.n_layers, 8, cfg.n_kv_heads, cfg.head_dim, DEV)
    kvc = PagedKVCache(cfg.n_layers, 8, cfg.n_kv_heads, cfg.head_dim, "cpu", dtype=torch.float32)
    rng = np.random.default_rng(0)
    toks = rng.integers(0, cfg.vocab, 43)
    bt = np.tile(np.arange(8, dtype=np.int32), (64, 1))
    pos = np.arange(40)   # longer than the sliding window (24): windowed layers differ
    lg = gpu.forward(_batch(toks[:40], pos, bt[:40], DEV, [39]), kvg, ctx)
    lc = cpu.forward(_batch(toks[:40], pos, bt[:40], "cpu", [39]), kvc)
    cos = torch.nn.functional.cosine_similarity(lg.cpu().double(), lc.double(), dim=-1)
    assert float(cos.min()) > 0.999, cos
    for p in range(40, 43):
        lg = gpu.forward(_batch([toks[p]], [p], bt[:1], DEV, [0]), kvg, ctx)
        lc = cpu.forward(_batch([toks[p]], [p], bt[:1], "cpu", [0]), kvc)
        cos = torch.nn.functional.cosine_similarity(lg.cpu().double(), lc.double(), dim=-1)
        assert float(cos.min()) > 0.999, (p, cos)
    ctx.gemm.check()
