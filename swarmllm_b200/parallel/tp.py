"""Tensor parallelism inside a node (one process per GPU), fused with the GEMMs.

Column-parallel layers (q|k|v, gate|up) split their output rows: every rank
holds n_heads/W query heads, n_kv/W KV heads and ffn/W features, and keeps
the full (replicated) residual stream, so their input needs no gather.
Row-parallel layers (o_proj, down_proj) split K.  Their reduction is fused
into two kernels over NVLink peer memory, with no collective call:

* the Q4_K GEMM's epilogue stores every 128-column tile of its partial
  result straight into the receive buffer of the rank that owns those hidden
  columns (reduce-scatter by P2P stores, tile by tile), and its last CTA
  raises a "GEMM done" flag on every rank;
* `tp_reduce_norm` (tp_comm.cu) sums the W partials of the owned columns,
  adds bias and residual, stores the new residual slice into every rank's
  copy (all-gather by P2P stores) with its sum of squares, and once every
  rank's slice of a row is in, applies the next RMSNorm to the whole row.

Per row-parallel layer each rank sends (W-1)/W of its partial result once and
its residual slice W-1 times; there is no all-gather of partials.

For few rows (decode: T * (W - 1) <= SWARMLLM_TP_LOCAL_ROWS, default 32) the
two cross-GPU hops of that scheme cost more than the bytes: the GEMM then
stores every tile into every rank's buffer and `tp_local_norm` sums all W
partials of every column locally (same order on every rank, so the
replicated residual stays identical), waiting only on the GEMM-done flags.

Arena (CUDA-IPC mapped, identical offsets on every rank), in bytes:
  recv      [2][W][ws]      fp32 partials per source rank (2 alternating buffers)
  gemm flag [2][W]          u32 GEMM-done epochs, one word per source rank
  h         [2][t_max][H]   fp32 residual stream copies (call k writes k % 2)
  ss        [2][W*16][t_max] fp32 sums of squares per (rank, row slice)
  row flag  [W*16][t_max]   u32 epochs per (rank, row slice)
Local control words (int32[16]): [4b+0..2] done counter, signal epoch and
wait epoch of receive buffer b; [8] done counter and [9] epoch of the rows.
Between row-parallel calls k and k+1 the residual lives in h[k % 2]; a
forward makes an even number of calls, so it starts and ends in h[1], which
`h_view()` exposes as the model's residual stream.

Reference behaviour: the reference's TP splits heads and FFN columns
(split/executor.rs:3440 pre_split_for_tp) and all-reduces f32 partials over
the network per layer and phase (src/inference/allreduce.rs:63,413,620).
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from ..utils.ext import C


class _DevBuf:
    """Zero-copy torch view of device memory the arena owns."""

    def __init__(self, ptr: int, shape, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3}


class TpGroup:
    # Status codes of the waits (GEMM-done flags; +1: row-slice flags)
    CODE_REDUCE = 73
    MAX_SLICES = 16  # CTAs per row of tp_reduce_norm (tp_comm.cu tp_reduce_slices)
    # one-hop reduce (partials to every rank) while T * (W - 1) is at most this
    LOCAL_ROWS = int(os.environ.get("SWARMLLM_TP_LOCAL_ROWS", "32"))

    def __init__(self, rank: int, world: int, device, group=None, timeout_ns: int = 0):
        assert 1 <= world <= 8
        self.rank, self.world = rank, world
        self.device = torch.device(device)
        self.group = group
        self.base = None
        self.k = 0
        self.timeout_ns = int(timeout_ns)  # 0: the kernels' default deadline (1 s)

    def setup(self, ws_floats: int, t_max: int, hidden: int):
        """Allocate this rank's arena and map every peer's (collective)."""
        if self.base is not None:
            assert ws_floats <= self.ws_floats and t_max <= self.t_max and hidden == self.H
            return
        W = self.world
        assert hidden % (128 * W) == 0, "every rank must own whole 128-column tiles"
        self.H, self.t_max = int(hidden), int(t_max)
        self.ws_floats = int(ws_floats)
        al = lambda n: (int(n) + 255) // 256 * 256
        self.ws_bytes = al(self.ws_floats * 4)
        self.flag_off = 2 * W * self.ws_bytes
        self.h_off = al(self.flag_off + 2 * W * 4)
        self.h_bytes = self.t_max * self.H * 4
        self.ss_off = al(self.h_off + 2 * self.h_bytes)
        self.slots = W * self.MAX_SLICES
        self.rf_off = al(self.ss_off + 2 * self.slots * self.t_max * 4)
        nbytes = al(self.rf_off + self.slots * self.t_max * 4)
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

    def h_view(self) -> torch.Tensor:
        """The residual stream [t_max, H] fp32 (this rank's copy, buffer 1)."""
        ptr = self.base + self.h_off + self.h_bytes
        return torch.as_tensor(_DevBuf(ptr, (self.t_max, self.H)), device=self.device)

    def begin_forward(self):
        self.k = 0

    def local(self, T: int) -> bool:
        """Whether T rows take the one-hop reduce (every rank sums every column)."""
        return T * (self.world - 1) <= self.LOCAL_ROWS

    def row_parallel(self, lin, x: torch.Tensor, status: torch.Tensor, num_sms: int):
        """GEMM of a K-split Q4_K weight; each result tile goes to its owner rank."""
        b = self.k & 1
        W, r = self.world, self.rank
        own = self.base + (b * W) * self.ws_bytes
        dsts = [self.bases[o] + (b * W + r) * self.ws_bytes for o in range(W)]
        owner_tiles = 0 if self.local(x.shape[0]) else self.H // 128 // W
        return C().qgemm_q4k_tc_tp(lin.packed, lin.rows, lin.K, x, status, num_sms, own,
                                   self.ws_bytes // 4, dsts, self.ctl[4 * b:], self.bases,
                                   self.flag_off + b * W * 4, r, owner_tiles, lin.fmt)

    def moe_partial(self, rows, wts, k: int, shared, shared_gate, T: int):
        """This rank's MoE output (its experts, its slice of the shared
        expert) stored into the column owners' receive slots, like a
        row-parallel GEMM's partials; reduce_norm sums them next."""
        b = self.k & 1
        W, r = self.world, self.rank
        own = self.base + (b * W) * self.ws_bytes
        dsts = [self.bases[o] + (b * W + r) * self.ws_bytes for o in range(W)]
        return C().moe_combine_tp(rows, wts, k, shared, shared_gate, T, self.H, own,
                                  self.ws_bytes // 4, dsts, self.ctl[4 * b:], self.bases,
                                  self.flag_off + b * W * 4, r, self.local(T))

    def reduce_norm(self, g, bias, w, out, eps: float, status: torch.Tensor, num_sms: int):
        """Residual += sum over ranks of the row-parallel result (+ bias), then
        out = RMSNorm(residual) * w; the residual ends up replicated."""
        k, W = self.k, self.world
        b = k & 1
        T = g.T
        assert T <= self.t_max
        if self.local(T):
            # residual updated in place in buffer 1 (h_view), where a forward
            # of slice-path calls also starts and ends
            C().tp_local_norm(g, self.h_view()[:T], bias, w, out, eps, W,
                              self.base + self.flag_off + b * W * 4, self.ctl, 4 * b + 2, 8,
                              status, self.CODE_REDUCE, self.timeout_ns)
            self.k += 1
            return
        C().tp_reduce_norm(g, bias, w, out, eps, self.H, self.rank, T, self.t_max, self.bases,
                           self.h_off + ((k + 1) & 1) * self.h_bytes,
                           self.h_off + b * self.h_bytes,
                           self.ss_off + b * self.slots * self.t_max * 4, self.rf_off,
                           self.base + self.flag_off + b * W * 4, self.ctl, 4 * b + 2, 8,
                           status, self.CODE_REDUCE, num_sms, self.timeout_ns)
        self.k += 1

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
