"""Mixture-of-experts FFN on the GPU: routing, dispatch, grouped expert GEMMs
on the tensor cores, combine (kernels in csrc/kernels/moe_tc.cu).

One MoE layer is six launches, all sized from host-side bounds so the whole
layer can be captured in a CUDA graph (the per-expert token counts stay on
the device):

    router GEMM  logits on the dense tensor-core GEMM (fp16 router weights)
    moe_topk     bias + top-k + routing weights + expert counts
    moe_plan     per-expert offsets and the (expert, token-tile) tile list
    moe_scatter  token rows -> expert-sorted rows (fp16 for Q4_K experts,
                 bf16 for MXFP4 experts), destination slot per row
    moe_gemm     gate|up grouped GEMM, SwiGLU epilogue -> H
    moe_gemm     down grouped GEMM, (+bias) rows stored at their (rank, slot)
    moe_combine  weighted sum over the k rows of a token (+ gated shared
                 expert), residual add, next RMSNorm

Reference: MoeFfn (src/inference/layers/moe.rs), expert GEMM kernels
vendor/candle/candle-kernels/src/moe/moe_gguf.cu:56 and moe_wmma_gguf.cu:191.
"""
from __future__ import annotations

import torch

from ..gguf import quants as Q
from ..utils.ext import C

FMT_Q4K, FMT_MXFP4 = 0, 1
EPI_SWIGLU, EPI_STORE = 0, 1


def _fmt_of(qtype: int) -> int:
    if qtype == Q.Q4_K:
        return FMT_Q4K
    if qtype == Q.MXFP4:
        return FMT_MXFP4
    raise NotImplementedError(f"expert weights of type {Q.TYPE_NAMES.get(qtype, qtype)}: the "
                              "grouped tensor-core GEMM takes Q4_K or MXFP4 experts")


def _repack(raw: torch.Tensor, fmt: int, rows: int, K: int, dev) -> torch.Tensor:
    """raw [E, rows, row_bytes] uint8 (GGUF blocks) -> packed [E, bytes] uint8."""
    E = raw.shape[0]
    nb = int(C().moe_packed_bytes(fmt, rows, K))
    out = torch.empty(E, nb, dtype=torch.uint8, device=dev)
    for e in range(E):
        if fmt == FMT_Q4K:
            C().q4k_repack(raw[e].contiguous(), rows, K, out[e])
        else:
            C().mxfp4_repack(raw[e].contiguous(), rows, K, out[e])
    return out


class MoeExperts:
    """Packed weights of one layer's experts (all of them, or the local slice
    [e0, e0 + n_local) under expert parallelism).

    gate|up rows are interleaved in groups of 16 (16 gate rows, then the
    matching 16 up rows) so that one warp of the GEMM epilogue holds both
    halves of a feature and applies the SwiGLU with one shuffle."""

    def __init__(self, gate, up, down, qtype: int, H: int, F: int, dev, e0: int = 0,
                 n_local: int | None = None, gate_b=None, up_b=None, down_b=None,
                 act_kind: int = 0, alpha: float = 1.702, limit: float = 7.0):
        assert F % 64 == 0, "expert FFN width must be a multiple of 64"
        self.fmt = _fmt_of(qtype)
        self.H, self.F = H, F
        E = gate.shape[0]
        n_local = E if n_local is None else n_local
        self.e0, self.n_local = e0, n_local
        sl = slice(e0, e0 + n_local)
        rb_in = Q.nbytes(qtype, H)
        g = gate[sl].to(dev).reshape(n_local, F // 16, 16, rb_in)
        u = up[sl].to(dev).reshape(n_local, F // 16, 16, rb_in)
        gu = torch.stack([g, u], dim=2).reshape(n_local, 2 * F, rb_in)
        self.w_gu = _repack(gu, self.fmt, 2 * F, H, dev)
        d = down[sl].to(dev).reshape(n_local, H, Q.nbytes(qtype, F))
        self.w_down = _repack(d, self.fmt, H, F, dev)
        self.b_gu = None
        if gate_b is not None:
            bg = gate_b[sl].reshape(n_local, F // 16, 16)
            bu = up_b[sl].reshape(n_local, F // 16, 16)
            self.b_gu = torch.stack([bg, bu], dim=2).reshape(n_local, 2 * F).float().to(dev).contiguous()
        self.b_down = down_b[sl].float().to(dev).contiguous() if down_b is not None else None
        self.act_kind, self.alpha, self.limit = act_kind, alpha, limit
        self.x_dtype = torch.bfloat16 if self.fmt == FMT_MXFP4 else torch.float16

    @property
    def nbytes(self) -> int:
        return self.w_gu.numel() + self.w_down.numel()


class MoeWorkspace:
    """Routing and dispatch buffers for up to `max_tokens` tokens."""

    def __init__(self, dev, max_tokens: int, H: int, F: int, E: int, k: int, x_dtype,
                 num_sms: int, max_pairs: int | None = None, ep=None):
        self.E, self.k, self.H, self.F = E, k, H, F
        P = max_pairs or max_tokens * k
        self.P = P
        i32 = dict(dtype=torch.int32, device=dev)
        self.ids = torch.zeros(max_tokens * k, **i32)
        self.wts = torch.zeros(max_tokens * k, dtype=torch.float32, device=dev)
        self.counts = torch.zeros(E, **i32)  # kept zero between layers by moe_plan
        self.offsets = torch.zeros(E + 1, **i32)
        self.cursor = torch.zeros(E, **i32)
        self.max_tiles = int(C().moe_max_tiles(P, E, 16))
        self.tiles = torch.zeros(self.max_tiles, 4, **i32)
        self.n_tiles = torch.zeros(1, **i32)
        self.ret = torch.zeros(P, **i32)
        self.xs = torch.zeros(P, H, dtype=x_dtype, device=dev)
        self.h = torch.zeros(P, F, dtype=x_dtype, device=dev)
        self.rows = torch.zeros(max_tokens * k, H, dtype=torch.float32, device=dev)
        self.status = torch.zeros(8, **i32)
        self.num_sms = num_sms
        if ep is not None:  # owner side: rows from every rank
            ep.setup(P, H, E, x_dtype)
            rows = ep.world * P
            self.ep_tiles = torch.zeros(int(C().moe_max_tiles(rows, ep.world * ep.e_loc, 16)),
                                        4, **i32)
            self.ep_h = torch.zeros(rows, F, dtype=x_dtype, device=dev)

    def check(self):
        s = self.status.cpu().tolist()
        if s[0]:
            raise RuntimeError(f"MoE kernel reported a timed-out wait: code {s[0]} block {s[1]} "
                               f"detail {s[2]},{s[3]}")
        if s[6]:
            raise RuntimeError(f"MoE tile list overflow: {s[6]} tiles")


def moe_route(x: torch.Tensor, router, router_b: torch.Tensor | None, ws: MoeWorkspace,
              gemm, softmax_after_topk: bool = True, mode: int | None = None,
              sel_b: torch.Tensor | None = None, norm: bool = True, scale: float = 1.0):
    """Router logits (QLinear on `gemm`) -> top-k ids / weights / counts in ws.
    mode: 0 softmax over all experts, 1 top-k then softmax (the default from
    `softmax_after_topk`), 2 sigmoid scores chosen with the selection bias
    `sel_b`, renormalised over the k when `norm`, times `scale`."""
    T = x.shape[0]
    lg = router(x, gemm)
    m = mode if mode is not None else (1 if softmax_after_topk else 0)
    C().moe_topk(lg, router_b, T, ws.E, ws.k, m, sel_b, norm, float(scale), ws.ids, ws.wts,
                 ws.counts)


def moe_experts(x: torch.Tensor, experts: MoeExperts, ws: MoeWorkspace, residual: torch.Tensor,
                norm_w: torch.Tensor | None, out: torch.Tensor | None, eps: float, shared=None,
                shared_gate=None):
    """Dispatch the routed rows, run the experts, combine into the residual
    (+ shared expert); out = RMSNorm(residual) * norm_w when out is given."""
    T = x.shape[0]
    E, k = ws.E, ws.k
    P = T * k
    c = C()
    N = int(c.moe_tok_tile(P, E))
    c.moe_plan(ws.counts, E, N, ws.offsets, ws.cursor, ws.tiles, ws.n_tiles, ws.status)
    c.moe_scatter(x, ws.ids[:P], k, ws.cursor, ws.xs, ws.ret, 0)
    ex = experts
    c.moe_gemm(ex.fmt, EPI_SWIGLU, ex.w_gu, 2 * ex.F, ex.H, ws.xs, N, ws.tiles, ws.n_tiles,
               ex.b_gu, 2 * ex.F, ws.h, ex.act_kind, ex.alpha, ex.limit, [], 0, None,
               ws.num_sms, ws.status)
    c.moe_gemm(ex.fmt, EPI_STORE, ex.w_down, ex.H, ex.F, ws.h, N, ws.tiles, ws.n_tiles,
               ex.b_down, ex.H, None, 0, 0.0, 0.0, [ws.rows.data_ptr()], ex.H, ws.ret,
               ws.num_sms, ws.status)
    c.moe_combine(ws.rows, ws.wts, k, shared, shared_gate, residual, norm_w, out, eps)


def moe_experts_ep(x: torch.Tensor, experts: MoeExperts, ws: "MoeWorkspace", ep,
                   residual: torch.Tensor, norm_w: torch.Tensor | None, out: torch.Tensor | None,
                   eps: float, shared=None, shared_gate=None):
    """moe_experts with the experts split over the ranks of `ep`
    (parallel/ep.py): P2P dispatch, grouped GEMMs on this rank's experts over
    every rank's rows, P2P combine from the down-projection epilogue."""
    T = x.shape[0]
    k = ws.k
    P = T * k
    c = C()
    ex = experts
    c.ep_dispatch(x, ws.ids[:P], k, ws.counts, ws.E, ep.e_loc, ep.cap, ws.cursor, ep.bases,
                  ep.rank, ep.x_bf16, ep.ctl)
    c.ep_wait(ep.base, ep.world, ep.cap, ep.H, ep.e_loc, 0, ep.ctl, ws.status)
    N = int(c.moe_tok_tile(P * ep.world, ep.e_loc))
    c.ep_plan_owner(ep.base, ep.world, ep.cap, ep.H, ep.e_loc, N, ws.ep_tiles, ws.n_tiles,
                    ws.status)
    c.moe_gemm(ex.fmt, EPI_SWIGLU, ex.w_gu, 2 * ex.F, ex.H, ep.recv_x, N, ws.ep_tiles, ws.n_tiles,
               ex.b_gu, 2 * ex.F, ws.ep_h, ex.act_kind, ex.alpha, ex.limit, [], 0, None,
               ws.num_sms, ws.status)
    c.moe_gemm(ex.fmt, EPI_STORE, ex.w_down, ex.H, ex.F, ws.ep_h, N, ws.ep_tiles, ws.n_tiles,
               ex.b_down, ex.H, None, 0, 0.0, 0.0, ep.comb_ptrs, ex.H, ep.recv_ret, ws.num_sms,
               ws.status, sig_ctl=ep.ctl[3:], sig_bases=ep.bases,
               sig_flag_off=ep.off["flags_c"], sig_rank=ep.rank)
    c.ep_wait(ep.base, ep.world, ep.cap, ep.H, ep.e_loc, 1, ep.ctl, ws.status)
    c.moe_combine(ep.comb, ws.wts, k, shared, shared_gate, residual, norm_w, out, eps)


def moe_experts_tp(x: torch.Tensor, experts: MoeExperts, ws: MoeWorkspace, tp, shared=None,
                   shared_gate=None):
    """The experts under tensor parallelism (parallel/tp.py): every rank of the
    group holds every token and experts [e0, e0 + n_local); it runs its own
    (token, k) pairs only and stores its share of the output into the column
    owners' buffers.  Returns the GemmOut that tp.reduce_norm sums."""
    T = x.shape[0]
    k = ws.k
    P = T * k
    c = C()
    ex = experts
    c.moe_localize(ws.ids[:P], ws.wts[:P], ws.counts, ws.E, ex.e0, ex.n_local)
    N = int(c.moe_tok_tile(P, ex.n_local))
    c.moe_plan(ws.counts, ex.n_local, N, ws.offsets, ws.cursor, ws.tiles, ws.n_tiles, ws.status)
    c.moe_scatter(x, ws.ids[:P], k, ws.cursor, ws.xs, ws.ret, 0)
    c.moe_gemm(ex.fmt, EPI_SWIGLU, ex.w_gu, 2 * ex.F, ex.H, ws.xs, N, ws.tiles, ws.n_tiles,
               ex.b_gu, 2 * ex.F, ws.h, ex.act_kind, ex.alpha, ex.limit, [], 0, None,
               ws.num_sms, ws.status)
    c.moe_gemm(ex.fmt, EPI_STORE, ex.w_down, ex.H, ex.F, ws.h, N, ws.tiles, ws.n_tiles,
               ex.b_down, ex.H, None, 0, 0.0, 0.0, [ws.rows.data_ptr()], ex.H, ws.ret,
               ws.num_sms, ws.status)
    return tp.moe_partial(ws.rows, ws.wts, k, shared, shared_gate, T)


def moe_ffn(x, experts, router, router_b, ws, gemm, residual, norm_w, out, eps,
            softmax_after_topk: bool = True, shared=None, shared_gate=None, **route):
    """Routing + experts + combine in one call (no shared expert between);
    `route`: moe_route's mode / sel_b / norm / scale."""
    moe_route(x, router, router_b, ws, gemm, softmax_after_topk, **route)
    moe_experts(x, experts, ws, residual, norm_w, out, eps, shared, shared_gate)
