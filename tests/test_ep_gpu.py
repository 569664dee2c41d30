"""Expert parallelism over peer memory (2 GPUs): every rank's MoE output with
the experts split over the ranks equals the single-GPU MoE with all experts.
Skipped with fewer than two GPUs."""
import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, fmt):
    import torch.distributed as dist
    from swarmllm_b200.gguf import quants as Q
    from swarmllm_b200.ops.linear import GemmWorkspace, QLinear
    from swarmllm_b200.ops.moe import (MoeExperts, MoeWorkspace, moe_experts, moe_experts_ep,
                                       moe_route)
    from swarmllm_b200.parallel.ep import EpGroup
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dev = torch.device(f"cuda:{rank}")
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    try:
        qt = Q.MXFP4 if fmt == "mxfp4" else Q.Q4_K
        E, k, H, F = 8, 2, (320 if fmt == "mxfp4" else 512), 256
        rng = np.random.default_rng(7)  # same weights on every rank

        def exp(rows, K):
            w = rng.standard_normal((E, rows, K), dtype=np.float32) * 0.05
            return torch.from_numpy(np.stack([Q.quantize(w[e], qt) for e in range(E)]))

        g, u, d = exp(F, H), exp(F, H), exp(H, F)
        ep = EpGroup(rank, world, dev)
        ex_loc = MoeExperts(g, u, d, qt, H, F, dev, e0=rank * (E // world), n_local=E // world)
        ex_all = MoeExperts(g, u, d, qt, H, F, dev)
        wr = rng.standard_normal((E, H), dtype=np.float32) * 0.2
        router = QLinear(torch.from_numpy(Q.quantize(wr, Q.F32)), Q.F32, E, H, dev, f32_as_f16=True)
        nsm = torch.cuda.get_device_properties(dev).multi_processor_count
        maxT = 16
        ws_ep = MoeWorkspace(dev, maxT, H, F, E, k, ex_loc.x_dtype, nsm, ep=ep)
        ws_ref = MoeWorkspace(dev, maxT, H, F, E, k, ex_all.x_dtype, nsm)
        gws = GemmWorkspace(dev, maxT, E)
        xr = np.random.default_rng(100 + rank)
        for call, T in enumerate((5 + 4 * rank, 16 - rank)):
            x = torch.from_numpy(xr.standard_normal((T, H), dtype=np.float32)).half().to(dev)
            r0 = torch.from_numpy(xr.standard_normal((T, H), dtype=np.float32)).to(dev)
            r_ep, r_ref = r0.clone(), r0.clone()
            moe_route(x, router, None, ws_ep, gws)
            moe_experts_ep(x, ex_loc, ws_ep, ep, r_ep, None, None, 1e-5)
            moe_route(x, router, None, ws_ref, gws)
            moe_experts(x, ex_all, ws_ref, r_ref, None, None, 1e-5)
            torch.cuda.synchronize(dev)
            ws_ep.check()
            assert torch.equal(ws_ep.ids[:T * k], ws_ref.ids[:T * k])
            rel = float((r_ep - r_ref).norm() / (r_ref - r0).norm())
            assert rel < 1e-5, (rank, call, rel)
        ep.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fmt", ["mxfp4", "q4k"])
def test_ep_matches_single_gpu(fmt):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    mp.spawn(_worker, args=(2, _free_port(), fmt), nprocs=2, join=True)
