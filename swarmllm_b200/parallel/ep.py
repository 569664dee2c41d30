"""Expert parallelism across the GPUs of one node (one process per GPU).

Attention and the dense layers are replicated (data parallel: every rank
serves its own requests); the routed experts of every MoE layer are split,
rank r owning experts [r*E/W, (r+1)*E/W).  Tokens travel to their experts
and results come back through peer-mapped device memory written by our own
kernels (csrc/kernels/ep_comm.cu): the dispatch is fused with routing/top-k
output and the combine with the down-projection GEMM's epilogue -- no NCCL
collective on this path, no host synchronisation, CUDA-graph capturable.

Every rank must run the same sequence of MoE layers (same steps), as with
any collective; the engine's lockstep over identical batch shapes gives that.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..utils.ext import C

_DT = {torch.bfloat16: "bf16", torch.float16: "f16"}


class EpGroup:
    def __init__(self, rank: int, world: int, device, group=None):
        assert 1 <= world <= 8, "expert parallelism over 1..8 GPUs of one node"
        self.rank, self.world = rank, world
        self.device = torch.device(device)
        self.group = group
        self.base = None

    def setup(self, cap: int, H: int, E: int, x_dtype):
        """Allocate this rank's arena and map every peer's (collective)."""
        if self.base is not None:
            assert (cap, H, E) == (self.cap, self.H, self.E), "EP arena already sized differently"
            return
        assert E % self.world == 0, "experts must divide evenly over the ranks"
        c = C()
        self.cap, self.H, self.E, self.e_loc = cap, H, E, E // self.world
        self.x_bf16 = x_dtype == torch.bfloat16
        nbytes = int(c.ep_arena_bytes(self.world, cap, H, self.e_loc))
        with torch.cuda.device(self.device):
            self.base, handle = c.ep_arena_alloc(nbytes)
        handles = [None] * self.world
        dist.all_gather_object(handles, handle, group=self.group)
        with torch.cuda.device(self.device):
            self.bases = [self.base if i == self.rank else int(c.ep_arena_open(handles[i]))
                          for i in range(self.world)]
        o = c.ep_arena_offsets(self.world, cap, H, self.e_loc)
        self.off = dict(zip(("recv_x", "recv_ret", "recv_cnt", "comb", "flags_d", "flags_c"), o))
        d = self.device.index or 0
        self.recv_x = c.ep_view(self.base, o[0], [self.world * cap, H], _DT[x_dtype], d)
        self.recv_ret = c.ep_view(self.base, o[1], [self.world * cap], "i32", d)
        self.comb = c.ep_view(self.base, o[3], [cap, H], "f32", d)
        self.comb_ptrs = [b + o[3] for b in self.bases]
        self.ctl = torch.zeros(16, dtype=torch.int32, device=self.device)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)

    def close(self):
        if self.base is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        c = C()
        for i, b in enumerate(self.bases):
            c.ep_arena_close(b, i == self.rank)
        self.base = None
