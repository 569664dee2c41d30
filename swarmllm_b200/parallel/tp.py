"""Tensor parallelism inside a node (one process per GPU), fused with the GEMMs.

Column-parallel layers (q|k|v, gate|up) split their output rows: every rank
holds n_heads/W query heads, n_kv/W KV heads and ffn/W features, and keeps
the full (replicated) residual stream, so their input needs no gather.
Row-parallel layers (o_proj, down_proj) split K; instead of an all-reduce
call, the Q4_K GEMM's own epilogue pushes its fp32 partial tiles over NVLink
into every rank's receive buffer (peer stores) and its last CTA raises a flag
on every rank (qgemm_tc.cu); the residual-add + RMSNorm epilogue then reads
the sum over the ranks' partials while it reads the GEMM result (GemmOut with
n_src ranks).  Two receive buffers alternate between consecutive row-parallel
GEMMs: a rank can only write buffer b again after every rank has read it
(each rank's next GEMM on b comes after its own wait on the GEMM in between).

Reference behaviour: the reference's TP splits heads and FFN columns
(split/executor.rs:3440 pre_split_for_tp) and all-reduces f32 partials over
the network per layer and phase (R27, src/network tp all-reduce).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..utils.ext import C


class TpGroup:
    def __init__(self, rank: int, world: int, device, group=None):
        assert 1 <= world <= 8
        self.rank, self.world = rank, world
        self.device = torch.device(device)
        self.group = group
        self.base = None
        self.buf = 0

    def setup(self, ws_floats: int):
        """Allocate this rank's receive buffers and map every peer's (collective)."""
        if self.base is not None:
            assert ws_floats <= self.ws_floats
            return
        W = self.world
        self.ws_floats = int(ws_floats)
        self.ws_bytes = (self.ws_floats * 4 + 255) // 256 * 256
        self.flag_off = 2 * W * self.ws_bytes
        nbytes = self.flag_off + 2 * W * 4 + 256
        c = C()
        with torch.cuda.device(self.device):
            self.base, handle = c.ep_arena_alloc(nbytes)
        handles = [None] * W
        dist.all_gather_object(handles, handle, group=self.group)
        with torch.cuda.device(self.device):
            self.bases = [self.base if i == self.rank else int(c.ep_arena_open(handles[i]))
                          for i in range(W)]
        self.ctl = torch.zeros(16, dtype=torch.int32, device=self.device)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)

    def begin_forward(self):
        self.buf = 0

    def row_parallel(self, lin, x: torch.Tensor, status: torch.Tensor, num_sms: int):
        """GEMM of a K-split Q4_K weight whose result is summed over the group."""
        b = self.buf
        self.buf ^= 1
        W, r = self.world, self.rank
        own = self.base + (b * W) * self.ws_bytes
        dsts = [self.bases[o] + (b * W + r) * self.ws_bytes for o in range(W)]
        ctl = self.ctl[4 * b:]
        g = C().qgemm_q4k_tc_tp(lin.packed, lin.rows, lin.K, x, status, num_sms, own,
                                self.ws_bytes // 4, dsts, ctl, self.bases,
                                self.flag_off + b * W * 4, r)
        C().flag_wait(self.base + self.flag_off + b * W * 4, W, ctl, 2, status, 71 + b)
        return g

    def close(self):
        if self.base is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        c = C()
        for i, b in enumerate(self.bases):
            c.ep_arena_close(b, i == self.rank)
        self.base = None


def split_rows(t: torch.Tensor, qt: int, shape, r0: int, r1: int) -> torch.Tensor:
    """Rows [r0, r1) of a GGML matrix given as raw bytes."""
    rows = shape[0]
    return t.view(rows, -1)[r0:r1].reshape(-1)


def split_cols(t: torch.Tensor, qt: int, shape, c0: int, c1: int) -> torch.Tensor:
    """Columns [c0, c1) of a GGML matrix (block-aligned) given as raw bytes."""
    from ..gguf import quants as Q
    rows, K = shape
    bv, bb = Q.BLOCK[qt]
    assert c0 % bv == 0 and c1 % bv == 0, "column split must align with quant blocks"
    return t.view(rows, K // bv, bb)[:, c0 // bv:c1 // bv].reshape(-1)
