"""Tensor-parallel reduce cost, one row-parallel layer (torchrun, N GPUs):

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m swarmllm_b200.parallel.tp_microbench

Times, per call, on the 70B down projection split N ways (K = 28672 / N):
the local Q4_K GEMM alone, the GEMM plus the single-GPU residual+RMSNorm
epilogue, and the row-parallel GEMM (owner-routed partial stores) plus the
fused reduce / residual / RMSNorm / all-gather kernel.  CUDA events over 50
calls, rank 0 prints (the ranks run in lockstep through the reduce's flags).
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
    for T in (1, 2, 8, 32):
        x = torch.randn(T, K, device=dev).half()
        out = torch.zeros(T, H, dtype=torch.float16, device=dev)

        def local():
            C().epi_residual_rmsnorm(lin(x, ws), h[:T], None, nw, out, 1e-5)

        def tpcall():
            tp.begin_forward()
            for _ in range(2):
                g = tp.row_parallel(lin, x, ws.status, ws.num_sms)
                tp.reduce_norm(g, None, nw, out, 1e-5, ws.status, ws.num_sms)
        res = {}
        for name, fn, per in (("gemm", lambda: lin(x, ws), 1), ("local gemm+epilogue", local, 1),
                              ("tp gemm+reduce", tpcall, 2)):
            for _ in range(5):
                fn()
            torch.cuda.synchronize()
            dist.barrier()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(50):
                fn()
            b.record()
            torch.cuda.synchronize()
            res[name] = a.elapsed_time(b) / 50 / per * 1000
        st = ws.status.cpu().tolist()
        if rank == 0:
            print(f"W={world} T={T} K={K}: " + ", ".join(f"{k} {v:.1f} us" for k, v in res.items())
                  + f"  status {st[0]}", flush=True)
    dist.barrier()
    tp.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
