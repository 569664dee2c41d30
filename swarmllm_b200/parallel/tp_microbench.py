"""Tensor-parallel reduce cost, one row-parallel layer (torchrun, N GPUs):

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m swarmllm_b200.parallel.tp_microbench

Times, per call, on the 70B down projection split N ways (K = 28672 / N):
the local Q4_K GEMM alone, the GEMM plus the single-GPU residual+RMSNorm
epilogue, the row-parallel GEMM (owner-routed partial stores) alone, and the
row-parallel GEMM plus the fused reduce / residual / RMSNorm / all-gather
kernel.  Each is captured 20 times in one CUDA graph (as the engine replays
its decode step), so the device time excludes host launch overhead; CUDA
events over 10 replays, rank 0 prints (the ranks run in lockstep through the
reduce's flags).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def main():
    from ..gguf import quants as Q
    from ..models.weights import _random_blocks_device
    from ..ops.linear import GemmWorkspace, QLinear, stream_k_floats
    from ..utils.ext import C
    from .pipeline import init_distributed
    from .tp import TpGroup
    init_distributed("nccl", timeout_s=300)
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device(f"cuda:{rank}")
    H, K = 8192, 28672 // world
    lin = QLinear(_random_blocks_device("w", (H, K), Q.Q4_K, 1, 0.02, dev), Q.Q4_K, H, K, dev)
    tp = TpGroup(rank, world, dev)
    ws = GemmWorkspace(dev, 64, H)
    tp.setup(stream_k_floats(64, H, ws.num_sms), 64, H)
    nw = torch.ones(H, device=dev)
    h = torch.zeros(64, H, device=dev)
    reps = 20

    def timed(fn):
        tp.begin_forward()
        for _ in range(4):                 # warm-up, eager (an even number of calls)
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        graph = torch.cuda.CUDAGraph()
        tp.begin_forward()
        with torch.cuda.graph(graph):
            for _ in range(reps):
                fn()
        torch.cuda.synchronize()
        dist.barrier()
        graph.replay()
        torch.cuda.synchronize()
        dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(10):
            graph.replay()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / (10 * reps) * 1000

    res = {}
    cases = {}
    for T in (1, 2, 8, 32):
        x = torch.randn(T, K, device=dev).half()
        out = torch.zeros(T, H, dtype=torch.float16, device=dev)

        def local(x=x, out=out, T=T):
            C().epi_residual_rmsnorm(lin(x, ws), h[:T], None, nw, out, 1e-5)

        def tp_call(x=x, out=out):
            g = tp.row_parallel(lin, x, ws.status, ws.num_sms)
            tp.reduce_norm(g, None, nw, out, 1e-5, ws.status, ws.num_sms)   # advances tp.k

        def tp_gemm(x=x):
            tp.row_parallel(lin, x, ws.status, ws.num_sms)
            tp.k += 1
        cases[T] = tp_gemm
        res[T] = {"gemm": timed(lambda x=x: lin(x, ws)), "local gemm+epilogue": timed(local),
                  "tp gemm+reduce": timed(tp_call)}
    # GEMMs without reduces run the done-flag epochs ahead of the reduce's
    # wait epoch (a later reduce would no longer wait): measured last
    for T in (1, 2, 8, 32):
        res[T]["tp gemm"] = timed(cases[T])
    st = ws.status.cpu().tolist()
    if rank == 0:
        for T, r in res.items():
            print(f"W={world} T={T} K={K}: " + ", ".join(f"{k} {v:.1f} us" for k, v in r.items())
                  + f"  status {st[0]}", flush=True)
    dist.barrier()
    tp.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
