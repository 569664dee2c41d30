"""Timings of the native CPU kernels (csrc/native/cpu_*.cpp) on this host:

    python -m swarmllm_b200.utils.cpu_cases [qmatmul|attention|decode] ...

qmatmul    the quantized matmul on a 4096 x 4096 weight (Q4_K, Q6_K, Q8_0) at
           1, 8 and 32 tokens, against fp32 torch on the dequantized matrix;
           GB/s counts the weight bytes once
attention  decode attention (32 query heads, 8 KV heads, head_dim 128) over
           fp16 pages at 512 and 4096 keys, 1 and 8 sequences
decode     the engine's decode step on a random 8-layer 2048-wide Q4_K model,
           fp32 PyTorch path vs the native path (`cpu_native`)

Wall-clock medians (the kernels are synchronous); OpenMP uses every core
unless OMP_NUM_THREADS says otherwise.
"""
from __future__ import annotations

import sys
import time

import numpy as np
import torch


def _median_s(fn, n: int = 7) -> float:
    fn()
    ts = []
    for _ in range(n):
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
    ts.sort()
    return ts[len(ts) // 2]


def qmatmul_case():
    from swarmllm_b200 import _native
    from swarmllm_b200.gguf import quants as Q
    rows = K = 4096
    print(f"isa {_native.cpu_qmatmul_isa()}, {torch.get_num_threads()} threads")
    rng = np.random.default_rng(0)
    for qt in (Q.Q4_K, Q.Q6_K, Q.Q8_0):
        w = Q.random_quantized(rows, K, qt, rng=rng)
        for T in (1, 8, 32):
            x = rng.standard_normal((T, K), dtype=np.float32)
            s = _median_s(lambda: _native.cpu_qmatmul(w, qt, rows, K, x))
            print(f"qmatmul {Q.TYPE_NAMES[qt]} T={T}: {s * 1e3:.2f} ms, "
                  f"{w.nbytes / s / 1e9:.1f} GB/s of weights")
    wf = torch.randn(rows, K)
    for T in (1, 8, 32):
        x = torch.randn(T, K)
        s = _median_s(lambda: x @ wf.T)
        print(f"fp32 torch T={T}: {s * 1e3:.2f} ms")


def attention_case():
    from swarmllm_b200 import _native
    nq, nkv, d, ps = 32, 8, 128, 16
    for L in (512, 4096):
        for N in (1, 8):
            pages = (L + ps - 1) // ps
            K = torch.randn(N * pages, nkv, ps, d).half().numpy()
            V = torch.randn(N * pages, nkv, ps, d).half().numpy()
            bt = np.arange(N * pages, dtype=np.int32).reshape(N, pages)
            lens = np.full(N, L, np.int32)
            q = np.random.default_rng(0).standard_normal((N, nq, d), dtype=np.float32)
            s = _median_s(lambda: _native.cpu_paged_attention(q, K, V, bt, lens, 0.088))
            kv_bytes = 2 * N * L * nkv * d * 2
            print(f"attention keys={L} seqs={N}: {s * 1e3:.2f} ms, {kv_bytes / s / 1e9:.1f} GB/s of KV")


def decode_case():
    from swarmllm_b200.engine import LLMEngine
    from swarmllm_b200.engine.engine import EngineConfig
    from swarmllm_b200.engine.sampling import SamplingParams
    from swarmllm_b200.models.config import ModelConfig
    from swarmllm_b200.models.weights import RandomSource
    cfg = ModelConfig(name="cpu-8l-2048", arch="llama", n_layers=8, hidden=2048, n_heads=16,
                      n_kv_heads=4, head_dim=128, ffn=8192, vocab=32000, weight_qtype="Q4_K",
                      embed_qtype="Q4_K", output_qtype="Q6_K", rope_theta=500000.0)
    src = RandomSource(cfg, seed=0)
    for native in (False, True):
        ec = EngineConfig(max_model_len=1024, max_running=8, kv_pages=512, cuda_graphs=False,
                          cpu_native=native, prefill_chunk=512, max_step_tokens=512,
                          prefix_cache=False)
        eng = LLMEngine.from_config(cfg, "cpu", ec, source=src)
        for B in (1, 4):
            prompts = [list(np.random.default_rng(i).integers(0, cfg.vocab, 128)) for i in range(B)]
            eng.generate(prompts, SamplingParams(max_tokens=2, temperature=0.0))
            t0 = time.perf_counter()
            eng.generate(prompts, SamplingParams(max_tokens=1, temperature=0.0))
            pre = time.perf_counter() - t0
            t0 = time.perf_counter()
            eng.generate(prompts, SamplingParams(max_tokens=33, temperature=0.0))
            step = (time.perf_counter() - t0 - pre) / 32
            print(f"decode native={native} batch={B}: {step * 1e3:.1f} ms/step, "
                  f"{B / step:.1f} tok/s (prefill of {B}x128 tokens {pre * 1e3:.0f} ms)")


def main(argv=None):
    argv = sys.argv[1:] if argv is None else argv
    which = argv or ["qmatmul", "attention", "decode"]
    for w in which:
        {"qmatmul": qmatmul_case, "attention": attention_case, "decode": decode_case}[w]()


if __name__ == "__main__":
    main()
