"""Standalone cases of the hot kernels, for profiling one kernel at a time:

    python -m swarmllm_b200.utils.kernel_cases \
        {qgemm|qgemm_sweep|mma_probe|qgemv|qgemv_o|dense|attn|attn_prefill|rmsnorm|swiglu|
         rope_kv|moe|delta|delta_decode|tree_rank|sample} [--time] [--qtype Q4_K|Q6_K|Q8_0]

Each case builds benchmark-sized operands on cuda:0 (inputs larger than the
126 MB L2 where memory traffic matters; tree_rank and sample use the real
logits size, which L2 holds), runs the kernel a few times and exits.  Under ncu, capture one launch after the warm-up ones, e.g.

    ncu --set full --clock-control none -k regex:qgemm_q4k -s 2 -c 1 \
        -o prof_qgemm python -m swarmllm_b200.utils.kernel_cases qgemm
"""
import sys
import math  # noqa: F401  (used by some cases)

import numpy as np  # noqa: F401
import torch

from swarmllm_b200.gguf import quants as Q
from swarmllm_b200.utils.ext import C

dev = "cuda:0"
_CASE = ["?"]  # name of the running case (for _time's report)

def _time(fn, n=50):
    """Median device time (us) of fn() over n calls after warm-up (inputs in L2 for the
    sampling cases: the logits a sampler reads were just written by the LM head)."""
    for _ in range(5):
        fn()
    ts = []
    for _ in range(n):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(); fn(); b.record(); torch.cuda.synchronize()
        ts.append(a.elapsed_time(b) * 1e3)
    ts.sort()
    print(f"{_CASE[0]}: median {ts[len(ts) // 2]:.1f} us over {n} calls")

def rand_q4k(rows, K, qt=Q.Q4_K):
    # random GGML blocks generated on the device (valid scales)
    from swarmllm_b200.models.weights import _random_blocks_device
    return _random_blocks_device("w", (rows, K), qt, 1, 0.02, dev)


def run_case(which: str, TIME: bool = False, qtype: str = "Q4_K") -> None:
    """Build one case's operands on cuda:0 and run its kernel a few times."""
    torch.manual_seed(0)
    _CASE[0] = which
    if which == "qgemm_sweep":  # the 70B projections at 1..2048 tokens: device time, GB/s, TFLOP/s
        from swarmllm_b200.ops.linear import GemmWorkspace, QLinear
        qt = Q.NAME_TO_TYPE[qtype]
        bv, bb = Q.BLOCK[qt]
        for rows, K, name in ((57344, 8192, "gate_up"), (8192, 28672, "down"), (8192, 8192, "o_proj")):
            lin = QLinear(rand_q4k(rows, K, qt), qt, rows, K, dev)
            for T in (1, 3, 8, 16, 32, 64, 128, 2048):
                ws = GemmWorkspace(dev, T, rows)
                x = torch.randn(T, K, device=dev).half()
                for _ in range(3):
                    lin(x, ws)
                torch.cuda.synchronize()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                n = 20 if T < 1024 else 5
                a.record()
                for _ in range(n):
                    lin(x, ws)
                b.record()
                torch.cuda.synchronize()
                us = a.elapsed_time(b) * 1000 / n
                print(f"{qtype} {name} {rows}x{K} T={T}: {us:8.1f} us  "
                      f"{rows * K * bb / bv / us / 1e3:6.0f} GB/s"
                      f"  {2 * rows * K * T / us / 1e6:7.1f} TFLOP/s", flush=True)
                ws.check()
    elif which == "mma_probe":   # tcgen05.mma issue cost per shape (one CTA per SM, clock64)
        sms = torch.cuda.get_device_properties(0).multi_processor_count
        iters = 2048
        for i, (ts, m, n) in enumerate(C().mma_probe_shapes()):
            cyc = torch.zeros(sms, dtype=torch.int64, device=dev)
            C().mma_probe(i, 64, cyc, 0)               # warm-up
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            C().mma_probe(i, iters, cyc, 0)
            b.record()
            torch.cuda.synchronize()
            per = float(cyc.float().median()) / (iters * 4)
            ns = a.elapsed_time(b) * 1e6 / (iters * 4)
            flop = 2.0 * m * n * 16 * sms / (ns * 1e-9) / 1e12
            print(f"{'TS' if ts else 'SS'} M={m:3d} N={n:3d} K=16: {per:6.1f} clk/MMA  "
                  f"{ns:6.1f} ns/MMA  {flop:7.1f} TFLOP/s (all SMs)", flush=True)
        # what a pipeline pays around its MMAs, every `grp` MMAs: a commit (no wait),
        # a commit + wait for completion, the same with 4 rotating accumulators,
        # or a 1500-clock pause of the issuing thread without any commit
        for i, (ts, m, n) in enumerate(C().mma_probe_shapes()):
            if not ts or n != 32:
                continue
            for grp in (4, 16, 48):
                for mode, spin, what in ((0, 0, "commit"), (1, 0, "commit+wait"),
                                         (3, 0, "commit+wait, 4 accumulators"),
                                         (4, 1500, "1500-clock pause")):
                    cyc = torch.zeros(sms, dtype=torch.int64, device=dev)
                    C().mma_probe(i, 512, cyc, grp, mode, spin)
                    torch.cuda.synchronize()
                    per = float(cyc.float().median()) / (512 * 4)
                    print(f"TS M={m:3d} N={n:3d}, every {grp:2d} MMAs {what}: {per:6.1f} clk/MMA "
                          f"({per * grp:7.1f} clk per group)", flush=True)
    elif which == "qgemm":       # Llama-3.3-70B gate|up at decode batch 32 (264 MB of weights)
        from swarmllm_b200.ops.linear import GemmWorkspace, QLinear
        rows, K, T = 57344, 8192, 32
        lin = QLinear(rand_q4k(rows, K), Q.Q4_K, rows, K, dev)
        ws = GemmWorkspace(dev, T, rows)
        x = torch.randn(T, K, device=dev).half()
        for _ in range(5): lin(x, ws)
    elif which == "qgemv":     # the same weights at decode batch 1 (CUDA-core GEMV path)
        from swarmllm_b200.ops.linear import GemmWorkspace, QLinear
        rows, K, T = 57344, 8192, 1
        lin = QLinear(rand_q4k(rows, K), Q.Q4_K, rows, K, dev)
        ws = GemmWorkspace(dev, T, rows)
        x = torch.randn(T, K, device=dev).half()
        for _ in range(5): lin(x, ws)
    elif which == "qgemv_o":   # the o projection at decode batch 1 (8192 x 8192, 38 MB)
        from swarmllm_b200.ops.linear import GemmWorkspace, QLinear
        rows, K, T = 8192, 8192, 1
        lin = QLinear(rand_q4k(rows, K), Q.Q4_K, rows, K, dev)
        ws = GemmWorkspace(dev, T, rows)
        x = torch.randn(T, K, device=dev).half()
        for _ in range(5): lin(x, ws)
    elif which == "dense":     # gpt-oss LM head (201088 x 2880 fp16, 1.16 GB) at batch 16
        from swarmllm_b200.ops.linear import GemmWorkspace, QLinear
        rows, K, T = 201088, 2880, 16
        w = (torch.randn(rows, K, device=dev) * 0.02).half()
        lin = QLinear(w.view(torch.uint8).reshape(-1), Q.F16, rows, K, dev)
        ws = GemmWorkspace(dev, T, rows)
        x = torch.randn(T, K, device=dev).half()
        for _ in range(5): lin(x, ws)
    elif which == "attn":      # decode batch 32, context 2300, 64 q / 8 kv heads, d 128 (300 MB KV)
        from swarmllm_b200.ops.attention import AttentionWorkspace, paged_attention
        B, L, nq, nkv, d, ps = 32, 2300, 64, 8, 128, 16
        ppseq = (L + ps - 1) // ps
        P = B * ppseq
        K = torch.randn(P, nkv, ps, d, device=dev).half(); V = torch.randn_like(K)
        bt = torch.arange(P, device=dev, dtype=torch.int32).view(B, ppseq)
        lens = torch.full((B,), L, dtype=torch.int32, device=dev)
        q = torch.randn(B, nq, d, device=dev).half()
        ws = AttentionWorkspace(dev, B, nq, nkv, d, L + 64)
        out = torch.empty_like(q)
        for _ in range(5):
            paged_attention(q, K, V, bt, lens, ws, out, L + 64, 1 / math.sqrt(d))
    elif which == "attn_prefill":  # 70B prefill chunk: 2048 causal positions of one sequence
        from swarmllm_b200.ops.attention import AttentionWorkspace, paged_attention
        T, nq, nkv, d, ps = 2048, 64, 8, 128, 16
        P = T // ps
        K = torch.randn(P, nkv, ps, d, device=dev).half(); V = torch.randn_like(K)
        bt = torch.arange(P, device=dev, dtype=torch.int32).view(1, P).expand(T, P).contiguous()
        lens = torch.arange(1, T + 1, dtype=torch.int32, device=dev)
        ppg = 128 // (nq // nkv)      # positions per row group
        row0 = torch.arange(0, T, ppg, dtype=torch.int32, device=dev)
        npos = torch.full_like(row0, ppg)
        q = torch.randn(T, nq, d, device=dev).half()
        ws = AttentionWorkspace(dev, T, nq, nkv, d, T)
        out = torch.empty_like(q)
        for _ in range(5):
            paged_attention(q, K, V, bt, lens, ws, out, T, 1 / math.sqrt(d), groups=(row0, npos, ppg))
    elif which == "rmsnorm":   # down projection + residual-add/RMSNorm epilogue, 2048-token chunk
        from swarmllm_b200.ops.linear import GemmWorkspace, QLinear
        rows, K, T = 8192, 28672, 2048
        lin = QLinear(rand_q4k(rows, K), Q.Q4_K, rows, K, dev)
        ws = GemmWorkspace(dev, T, rows)
        x = torch.randn(T, K, device=dev).half()
        h = torch.randn(T, rows, device=dev)
        w = torch.ones(rows, device=dev)
        out = torch.empty(T, rows, device=dev).half()
        for _ in range(5):
            C().epi_residual_rmsnorm(lin(x, ws), h, None, w, out, 1e-5)
        if TIME:   # the epilogue alone, over the last GEMM's partial sums
            g = lin(x, ws)
            _time(lambda: C().epi_residual_rmsnorm(g, h, None, w, out, 1e-5))
    elif which == "swiglu":    # gate|up projection + SwiGLU epilogue, 2048-token chunk
        from swarmllm_b200.ops.linear import GemmWorkspace, QLinear
        rows, K, T = 57344, 8192, 2048
        lin = QLinear(rand_q4k(rows, K), Q.Q4_K, rows, K, dev)
        ws = GemmWorkspace(dev, T, rows)
        x = torch.randn(T, K, device=dev).half()
        act = torch.empty(T, rows // 2, device=dev).half()
        for _ in range(5):
            C().epi_swiglu(lin(x, ws), None, rows // 2, 0, False, 0.0, 0.0, act)
        if TIME:   # the epilogue alone, over the last GEMM's partial sums
            g = lin(x, ws)
            _time(lambda: C().epi_swiglu(g, None, rows // 2, 0, False, 0.0, 0.0, act))
    elif which == "rope_kv":   # QKV projection + RoPE / paged-KV-append epilogue, 70B, 2048-token chunk
        from swarmllm_b200.ops.linear import GemmWorkspace, QLinear
        nq, nkv, d, ps, T, K = 64, 8, 128, 16, 2048, 8192
        rows = (nq + 2 * nkv) * d
        lin = QLinear(rand_q4k(rows, K), Q.Q4_K, rows, K, dev)
        ws = GemmWorkspace(dev, T, rows)
        x = torch.randn(T, K, device=dev).half()
        pos = torch.arange(T, dtype=torch.int32, device=dev)
        inv_freq = 1.0 / (500000.0 ** (torch.arange(0, d, 2, device=dev).float() / d))
        qo = torch.empty(T, nq, d, device=dev).half()
        kc = torch.zeros(T // ps, nkv, ps, d, device=dev).half(); vc = torch.zeros_like(kc)
        run = lambda g: C().epi_rope_kv(g, None, pos, pos, inv_freq, nq, nkv, d, d, False, 1.0, qo,
                                        kc, vc, ps, None, None, 0.0, None)
        for _ in range(5):
            run(lin(x, ws))
        if TIME:   # the epilogue alone, over the last GEMM's partial sums
            g = lin(x, ws)
            _time(lambda: run(g))
    elif which == "delta_decode":  # Qwen3-Next-style recurrent delta rule, decode batch 8, 32 v heads
        from swarmllm_b200.ops.linear import GemmWorkspace, QLinear
        B, nk, nv, D = 8, 16, 32, 128
        C_ = (2 * nk + nv) * D
        qkv = torch.randn(B, C_, device=dev)
        x = torch.randn(B, 2048, device=dev).half()
        wba = QLinear((torch.randn(2 * nv, 2048, device=dev) * 0.02).half().view(torch.uint8).reshape(-1), Q.F16, 2 * nv, 2048, dev)
        wz = QLinear((torch.randn(nv * D, 2048, device=dev) * 0.02).half().view(torch.uint8).reshape(-1), Q.F16, nv * D, 2048, dev)
        gba, gz = wba(x, GemmWorkspace(dev, B, 2 * nv)), wz(x, GemmWorkspace(dev, B, nv * D))
        A = -torch.rand(nv, device=dev); dtb = torch.rand(nv, device=dev)
        nw = torch.ones(D, device=dev)
        state = torch.randn(B + 1, nv, D, D, device=dev) * 0.01     # 16 MB of fp32 state
        seqs = torch.tensor([[i, 1, i, 100] for i in range(B)], dtype=torch.int32, device=dev)
        out = torch.zeros(B, nv * D, device=dev).half()
        run = lambda: C().delta_rule(qkv, nk, nv, D, gba, dtb, A, gz, nw, 1e-6, state, seqs, B, out)
        for _ in range(5):
            run()
        if TIME:
            _time(run)
    elif which == "tree_rank":  # drafter top-4 over a 128256 vocabulary, 32 sequences x width 4
        rows, V, W = 128, 128256, 4
        logits = torch.randn(rows, V, device=dev) * 3
        ids = torch.zeros(rows * W, dtype=torch.int32, device=dev)
        lp = torch.zeros(rows * W, device=dev)
        rk = torch.zeros(int(C().tree_rank_ws_floats(rows, V, W)), device=dev)
        for _ in range(5):
            C().tree_rank(logits, W, ids, lp, rk)
        if TIME:
            _time(lambda: C().tree_rank(logits, W, ids, lp, rk))
    elif which == "sample":     # temperature / top-k / top-p sampling of 32 rows over 128256 tokens
        rows, V = 32, 128256
        logits = torch.randn(rows, V, device=dev) * 3
        temp = torch.full((rows,), 0.8, device=dev)
        topk = torch.full((rows,), 40, dtype=torch.int32, device=dev)
        topp = torch.full((rows,), 0.95, device=dev)
        seeds = torch.arange(rows, dtype=torch.int64, device=dev)
        pos = torch.full((rows,), 100, dtype=torch.int32, device=dev)
        out = torch.zeros(rows, dtype=torch.int32, device=dev)
        for _ in range(5):
            C().sample(logits, temp, topk, topp, seeds, pos, out)
        if TIME:
            _time(lambda: C().sample(logits, temp, topk, topp, seeds, pos, out))
            topk.zero_()           # top-p alone: the whole-row mass path
            which = "sample (top_p only)"
            _time(lambda: C().sample(logits, temp, topk, topp, seeds, pos, out))
    elif which == "moe":       # gpt-oss-style experts (32 of 128, MXFP4), batch 64 tokens top-4
        from swarmllm_b200.ops.linear import GemmWorkspace, QLinear
        from swarmllm_b200.ops.moe import MoeExperts, MoeWorkspace, moe_ffn
        from swarmllm_b200.models.weights import _random_blocks_device
        E, k, H, F, T = 32, 4, 2880, 2880, 64
        g = _random_blocks_device("g", (E, F, H), Q.MXFP4, 1, 0.02, dev).view(E, F, -1)
        u = _random_blocks_device("u", (E, F, H), Q.MXFP4, 1, 0.02, dev).view(E, F, -1)
        dn = _random_blocks_device("d", (E, H, F), Q.MXFP4, 1, 0.02, dev).view(E, H, -1)
        ex = MoeExperts(g, u, dn, Q.MXFP4, H, F, dev, act_kind=1)
        wr = (torch.randn(E, H, device=dev) * 0.1).half()
        router = QLinear(wr.view(torch.uint8).reshape(-1), Q.F16, E, H, dev)
        ws = MoeWorkspace(dev, T, H, F, E, k, ex.x_dtype, 148)
        gws = GemmWorkspace(dev, T, E)
        x = torch.randn(T, H, device=dev).half()
        r = torch.zeros(T, H, device=dev)
        for _ in range(5): moe_ffn(x, ex, router, None, ws, gws, r, None, None, 1e-5)
    elif which == "delta":     # Qwen3-Next-style DeltaNet prefill: 4096 tokens, 16 k / 32 v heads
        from swarmllm_b200.ops.linear import GemmWorkspace, QLinear
        T, nk, nv, D = 4096, 16, 32, 128
        C_ = (2 * nk + nv) * D
        qkv = torch.randn(T, C_, device=dev)
        gws = GemmWorkspace(dev, T, 2 * nv)
        x = torch.randn(T, 2048, device=dev).half()
        wba = QLinear((torch.randn(2 * nv, 2048, device=dev) * 0.02).half().view(torch.uint8).reshape(-1), Q.F16, 2 * nv, 2048, dev)
        wz = QLinear((torch.randn(nv * D, 2048, device=dev) * 0.02).half().view(torch.uint8).reshape(-1), Q.F16, nv * D, 2048, dev)
        gws2 = GemmWorkspace(dev, T, nv * D)
        gba, gz = wba(x, gws), wz(x, gws2)
        A = -torch.rand(nv, device=dev); dtb = torch.rand(nv, device=dev)
        nw = torch.ones(D, device=dev)
        state = torch.zeros(2, nv, D, D, device=dev)
        seqs = torch.tensor([[0, T, 1, 0]], dtype=torch.int32, device=dev)
        oraw = torch.zeros(T, nv * D, device=dev); out = torch.zeros(T, nv * D, device=dev).half()
        for _ in range(3):
            C().delta_chunk(qkv, nk, nv, D, gba, dtb, A, gz, nw, 1e-6, state, seqs, 1, oraw, out)
        if TIME:
            _time(lambda: C().delta_chunk(qkv, nk, nv, D, gba, dtb, A, gz, nw, 1e-6, state, seqs, 1,
                                          oraw, out), n=10)
    torch.cuda.synchronize()
    print("ok", which)


def main(argv=None) -> None:
    argv = sys.argv[1:] if argv is None else argv
    qtype = argv[argv.index("--qtype") + 1] if "--qtype" in argv else "Q4_K"
    which = next((a for a in argv if not a.startswith("--") and a != qtype), "qgemm")
    run_case(which, "--time" in argv, qtype)


if __name__ == "__main__":
    main()
