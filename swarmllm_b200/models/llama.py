"""Llama-family decoder: GPU implementation (sm_100a kernels) and a CPU
implementation (PyTorch fp32) that doubles as the numerical oracle.

Both run a *flattened mixed batch*: N token rows from any number of sequences
(decode rows and prefill chunks together), each row with its own position,
KV slot, block-table row and visible length.  A model instance may hold only
a contiguous layer range (pipeline stage): the first stage embeds tokens, the
last applies the final norm + LM head; stages exchange the fp32 residual.

Per layer on the GPU (8 launches):
  qkv GEMM -> [bias + RoPE + q/k-norm + paged KV append]      (epi_rope_kv)
  paged attention (GQA, window, sinks)                          (decode_attn)
  o GEMM -> [residual add + RMSNorm(ffn_norm)]                  (epi_residual_rmsnorm)
  gate|up GEMM -> [SwiGLU]                                      (epi_swiglu)
  down GEMM -> [residual add + RMSNorm(next attn_norm)]         (epi_residual_rmsnorm)
Reference call stack: SplitModel::forward -> dense_layer
(src/inference/split/executor.rs:1095,3761), LayerWeights::attend
(src/inference/layers/mod.rs:5977).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

from ..gguf import quants as Q
from ..ops.attention import AttentionWorkspace, PagedKVCache, paged_attention
from ..ops.linear import GemmWorkspace, QLinear
from ..parallel.tp import split_cols, split_rows
from ..ops.moe import (MoeExperts, MoeWorkspace, moe_experts, moe_experts_ep, moe_experts_tp,
                       moe_route)
from ..utils.ext import C
from .config import ModelConfig, rope_inv_freq


@dataclass
class StepBatch:
    """Device (or CPU) tensors describing one forward's token rows."""
    tokens: torch.Tensor        # int32 [N]
    positions: torch.Tensor     # int32 [N]
    slots: torch.Tensor         # int32 [N]
    block_table: torch.Tensor   # int32 [N, max_pages]
    seq_lens: torch.Tensor      # int32 [N] visible keys per row
    sample_rows: torch.Tensor   # int64 [S]
    max_len: int                # max visible length (host int, for split planning)
    tree_mask: torch.Tensor | None = None   # uint64 [N] (as int64)
    tree_start: torch.Tensor | None = None  # int32 [N]
    groups: tuple | None = None             # (row0 int32[G], npos int32[G], positions/group)
    ssm_seqs: torch.Tensor | None = None    # int32 [S, 4] (row0, nrows, state slot, pos0): linear attention
    ssm_max_rows: int = 1                   # host hint: most rows of one sequence in this step
    lora_ids: torch.Tensor | None = None    # int32 [N] adapter index per row (-1: none)
    embed_rows: torch.Tensor | None = None  # int32 [n] rows whose embedding is given (images)
    embed_vals: torch.Tensor | None = None  # [n, hidden] those rows' embeddings


def _f32(t: torch.Tensor, qt: int, shape) -> torch.Tensor:
    """Decode a small F32/F16 tensor given as raw bytes."""
    arr = Q.dequantize(t.cpu().numpy().reshape(-1), qt).reshape(shape)
    return torch.from_numpy(np.ascontiguousarray(arr, dtype=np.float32))


class _GpuLayer:
    pass


class LlamaGPU:
    def __init__(self, cfg: ModelConfig, source, device, layer_range: tuple[int, int] | None = None,
                 kv_layer_offset: int | None = None, ep=None, tp=None):
        """`ep`: an EpGroup (parallel/ep.py) -- this rank then holds only its
        share of every MoE layer's experts and exchanges tokens with the
        other ranks inside each MoE layer.  `tp`: a TpGroup (parallel/tp.py)
        -- this rank holds n_heads/W query heads, n_kv/W KV heads and ffn/W
        FFN features; o_proj/down_proj partials are summed over the group by
        the GEMM epilogues."""
        unbuilt = [what for what, on in (
            ("layers without RoPE (llama4 iRoPE)", cfg.nope_every),
            ("q/k RMS normalisation without a weight (llama4)", cfg.qk_rms_plain),
            ("experts weighted on their input (llama4)", cfg.moe_weight_input),
            ("a residual multiplier (granite)", cfg.residual_scale)) if on]
        if unbuilt:
            raise NotImplementedError(f"{cfg.arch} on the GPU model: {', '.join(unbuilt)} not "
                                      "built in the kernels; the CPU model (device='cpu') runs it")
        self.cfg = cfg
        self.ep = ep
        self.tp = tp
        self.lora = None
        W = tp.world if tp else 1
        tr = tp.rank if tp else 0
        assert cfg.n_heads % W == 0 and cfg.ffn % W == 0
        self.n_q, self.ffn_loc = cfg.n_heads // W, cfg.ffn // W
        # KV heads of this rank's query heads: an even split, or -- with fewer KV
        # heads than ranks -- the one KV head its query heads share, replicated
        rep = cfg.n_heads // cfg.n_kv_heads
        self.kv0 = (tr * self.n_q) // rep
        self.n_kv = ((tr + 1) * self.n_q - 1) // rep + 1 - self.kv0
        assert cfg.n_kv_heads % W == 0 or (W % cfg.n_kv_heads == 0 and self.n_q <= rep), \
            "query heads of a rank must map onto whole KV heads"
        # linear-attention heads (gated DeltaNet), split by head
        if cfg.full_attn_interval:
            assert cfg.ssm_k_heads % W == 0 and cfg.ssm_v_heads % W == 0
        self.nk_loc, self.nv_loc = cfg.ssm_k_heads // W, cfg.ssm_v_heads // W
        if cfg.n_experts and tp is not None:
            assert cfg.n_experts % W == 0 and cfg.shared_expert_ffn % W == 0
        self.device = torch.device(device)
        lo, hi = layer_range or (0, cfg.n_layers)
        self.lo, self.hi = lo, hi
        self.first, self.last = lo == 0, hi == cfg.n_layers
        # KV caches are stage-local: layer lo of this stage is cache layer 0.
        self.kv_off = 0 if kv_layer_offset is None else kv_layer_offset
        dev = self.device
        H = cfg.hidden

        def get(name):
            return source.get(name, device=dev)

        def small(name):
            t, qt, shape = source.get(name)
            return _f32(t, qt, shape).to(dev)

        if self.first:
            t, qt, shape = get("token_embd.weight")
            self.embd, self.embd_type = t, qt
        self.layers = []
        n_attn = n_lin = 0
        for i in range(lo, hi):
            b = f"blk.{i}."
            L = _GpuLayer()
            L.attn_norm = small(b + "attn_norm.weight")
            L.ffn_norm = small(b + "ffn_norm.weight")
            L.linear = cfg.is_linear_attn(i)
            if L.linear:
                L.lin_idx = n_lin
                n_lin += 1
                self._load_deltanet(L, b, get, small)
            else:
                L.kv_idx = n_attn
                n_attn += 1
                d = cfg.head_dim
                qh = 2 * d if cfg.attn_output_gate else d
                kv_rows = (self.kv0 * d, (self.kv0 + self.n_kv) * d)
                shares = ((tr * self.n_q * qh, (tr + 1) * self.n_q * qh), kv_rows, kv_rows)
                rows = sum(z - a for a, z in shares)
                if cfg.fused_qkv:  # one q|k|v tensor: each part's rows at its offset
                    t, qt, shape = get(b + "attn_qkv.weight")
                    base = (0, cfg.n_heads * qh, cfg.n_heads * qh + cfg.kv_dim)
                    if W > 1:
                        t = torch.cat([split_rows(t, qt, shape, o + a, o + z)
                                       for o, (a, z) in zip(base, shares)])
                    L.wqkv = QLinear(t, qt, rows, H, dev)
                    L.qkv_bias = None
                    if cfg.attn_bias:
                        bq = small(b + "attn_qkv.bias")
                        L.qkv_bias = torch.cat([bq[o + a:o + z] for o, (a, z) in zip(base, shares)])
                else:
                    parts = [get(b + n) for n in ("attn_q.weight", "attn_k.weight", "attn_v.weight")]
                    pieces = [(split_rows(p[0], p[1], p[2], a, z) if W > 1 else p[0], p[1], z - a)
                              for p, (a, z) in zip(parts, shares)]
                    L.wqkv = QLinear.from_parts(pieces, H, dev)
                    L.qkv_bias = None
                    if cfg.attn_bias:
                        L.qkv_bias = torch.cat([small(b + n)[a:z] for n, (a, z) in
                                                zip(("attn_q.bias", "attn_k.bias", "attn_v.bias"),
                                                    shares)])
                t, qt, shape = get(b + "attn_output.weight")
                if W > 1:
                    t = split_cols(t, qt, shape, tr * self.n_q * d, (tr + 1) * self.n_q * d)
                L.wo = QLinear(t, qt, shape[0], self.n_q * d, dev)
                L.o_bias = small(b + "attn_output.bias") if cfg.has_out_bias else None
                L.post_attn_norm = small(b + "post_attention_norm.weight") if cfg.post_norms else None
                L.local_rope = bool(cfg.rope_local_theta) and cfg.is_swa(i)
                L.q_norm = small(b + "attn_q_norm.weight") if cfg.qk_norm else None
                L.k_norm = small(b + "attn_k_norm.weight") if cfg.qk_norm else None
                L.sinks = (small(b + "attn_sinks.weight")[tr * self.n_q:(tr + 1) * self.n_q]
                           .contiguous() if cfg.attn_sinks else None)
                L.window = cfg.sliding_window if cfg.is_swa(i) else 0
                L.gated = cfg.attn_output_gate
            L.experts = None
            L.sh_gu = L.sh_down = L.sh_gate = L.sel_b = None
            L.post_ffn_norm = small(b + "post_ffw_norm.weight") if cfg.post_norms else None
            if cfg.is_moe_layer(i):
                self._load_moe(L, b, get, small)
            else:
                F = self.ffn_loc
                if cfg.fused_gate_up:  # ffn_up holds gate rows [0, ffn) then up rows [ffn, 2 ffn)
                    u = get(b + "ffn_up.weight")
                    g = u
                    goff, uoff = 0, cfg.ffn
                else:
                    g, u = get(b + "ffn_gate.weight"), get(b + "ffn_up.weight")
                    goff = uoff = 0
                if W > 1 or cfg.fused_gate_up:
                    gp = split_rows(g[0], g[1], g[2], goff + tr * F, goff + (tr + 1) * F)
                    up = split_rows(u[0], u[1], u[2], uoff + tr * F, uoff + (tr + 1) * F)
                else:
                    gp, up = g[0], u[0]
                L.wgu = QLinear.from_parts([(gp, g[1], F), (up, u[1], F)], H, dev)
                t, qt, shape = get(b + "ffn_down.weight")
                if W > 1:
                    t = split_cols(t, qt, shape, tr * F, (tr + 1) * F)
                L.wdown = QLinear(t, qt, shape[0], F, dev)
                if W > 1:
                    assert L.wo.kind == "q4k" and L.wdown.kind == "q4k", \
                        "row-parallel layers run on the fused Q4_K tensor-core GEMM"
            self.layers.append(L)
        self.n_kv_layers, self.n_lin_layers = n_attn, n_lin
        self.next_norm = None
        if self.last:
            self.out_norm = small("output_norm.weight")
            name = "token_embd.weight" if cfg.tie_embeddings else "output.weight"
            t, qt, shape = get(name)
            self.head = QLinear(t, qt, shape[0], shape[1], dev)
        inv, self.attn_factor = rope_inv_freq(cfg)
        self.inv_freq = torch.from_numpy(inv).to(dev)
        inv_l, self.attn_factor_local = rope_inv_freq(cfg, local=True)
        self.inv_freq_local = torch.from_numpy(inv_l).to(dev)
        self.scale = cfg.softmax_scale
        self.act_kind = 2 if cfg.act == "gelu" else 0
        if tp is not None:
            assert not cfg.post_norms, "tensor parallelism covers the pre-norm families"

    def _load_deltanet(self, L, b, get, small):
        """Gated DeltaNet layer: in-projection (q|k|v), z gate, beta/decay
        projection, conv1d, decay parameters, gated norm, out-projection.
        Under tensor parallelism a rank holds nk/W key heads and the nv/W
        value heads that read them: its rows of q, k, v, z, beta and alpha,
        its conv channels and decay parameters, and its K-slice of the
        out-projection (row-parallel, reduced with the other ranks)."""
        cfg, dev, H = self.cfg, self.device, self.cfg.hidden
        nk, nv, dh = cfg.ssm_k_heads, cfg.ssm_v_heads, cfg.ssm_head_dim
        W, tr = (self.tp.world, self.tp.rank) if self.tp else (1, 0)
        nkl, nvl = self.nk_loc, self.nv_loc
        # channel ranges of this rank in the [q | k | v] projection / conv
        ch = [(tr * nkl * dh, (tr + 1) * nkl * dh),
              (nk * dh + tr * nkl * dh, nk * dh + (tr + 1) * nkl * dh),
              (2 * nk * dh + tr * nvl * dh, 2 * nk * dh + (tr + 1) * nvl * dh)]

        def rows_of(t, qt, shape, ranges):
            return t if W == 1 else torch.cat([split_rows(t, qt, shape, a, z) for a, z in ranges])
        t, qt, shape = get(b + "attn_qkv.weight")
        L.w_in = QLinear(rows_of(t, qt, shape, ch), qt, (2 * nkl + nvl) * dh, H, dev)
        t, qt, shape = get(b + "attn_gate.weight")
        L.w_z = QLinear(rows_of(t, qt, shape, [(tr * nvl * dh, (tr + 1) * nvl * dh)]), qt,
                        nvl * dh, H, dev)
        t, qt, shape = get(b + "ssm_ba.weight")
        L.w_ba = QLinear(rows_of(t, qt, shape, [(tr * nvl, (tr + 1) * nvl),
                                                (nv + tr * nvl, nv + (tr + 1) * nvl)]),
                         qt, 2 * nvl, H, dev, f32_as_f16=True)
        conv = small(b + "ssm_conv1d.weight")
        L.conv_w = (conv if W == 1 else torch.cat([conv[a:z] for a, z in ch])).contiguous()
        L.dt_bias = small(b + "ssm_dt.bias")[tr * nvl:(tr + 1) * nvl].contiguous()
        L.A = small(b + "ssm_a")[tr * nvl:(tr + 1) * nvl].contiguous()
        L.ssm_norm = small(b + "ssm_norm.weight")
        t, qt, shape = get(b + "ssm_out.weight")
        if W > 1:
            t = split_cols(t, qt, shape, tr * nvl * dh, (tr + 1) * nvl * dh)
        L.w_out = QLinear(t, qt, H, nvl * dh, dev)

    def linear_state_spec(self):
        """(n_layers, nv, dk, dv, conv_channels, conv_k) of this stage's
        linear-attention layers, or None."""
        if not self.n_lin_layers:
            return None
        c = self.cfg
        return (self.n_lin_layers, self.nv_loc, c.ssm_head_dim, c.ssm_head_dim,
                (2 * self.nk_loc + self.nv_loc) * c.ssm_head_dim, c.ssm_conv_kernel)

    def _load_moe(self, L, b, get, small):
        """Routed experts (+ router, + shared expert) of one layer."""
        cfg, dev = self.cfg, self.device
        E, F, H = cfg.n_experts, cfg.expert_ffn, cfg.hidden
        g, u, d = (get(b + n) for n in ("ffn_gate_exps.weight", "ffn_up_exps.weight",
                                         "ffn_down_exps.weight"))
        qt = g[1]
        rb_h, rb_f = Q.nbytes(qt, H), Q.nbytes(qt, F)
        biases = {}
        if cfg.arch == "gpt-oss":
            biases = dict(gate_b=small(b + "ffn_gate_exps.bias").cpu(),
                          up_b=small(b + "ffn_up_exps.bias").cpu(),
                          down_b=small(b + "ffn_down_exps.bias").cpu())
        ep = self.ep or self.tp   # experts split over the EP group or the TP group
        shard = dict(e0=ep.rank * (E // ep.world), n_local=E // ep.world) if ep else {}
        L.experts = MoeExperts(g[0].view(E, F, rb_h), u[0].view(E, F, rb_h),
                               d[0].view(E, H, rb_f), qt, H, F, dev, **shard,
                               act_kind=1 if cfg.swiglu_limit else 0, alpha=cfg.swiglu_alpha,
                               limit=cfg.swiglu_limit, **biases)
        del g, u, d
        t, rq, _ = get(b + "ffn_gate_inp.weight")
        L.router = QLinear(t, rq, E, H, dev, f32_as_f16=True)
        L.router_b = small(b + "ffn_gate_inp.bias") if cfg.arch == "gpt-oss" else None
        L.sel_b = (small(b + "exp_probs_b.bias") if cfg.moe_gating == "sigmoid" and cfg.moe_sel_bias
                   else None)
        L.sh_gu = L.sh_down = L.sh_gate = None
        if cfg.shared_expert_ffn:
            W, tr = (self.tp.world, self.tp.rank) if self.tp else (1, 0)
            gs, us = get(b + "ffn_gate_shexp.weight"), get(b + "ffn_up_shexp.weight")
            dq_t = get(b + "ffn_down_shexp.weight")[1]
            if W > 1 and cfg.shared_expert_ffn % (Q.BLOCK[dq_t][0] * W):
                # too narrow to split into whole quant blocks: rank 0 runs it alone
                W, tr = 1, 0
                if self.tp.rank != 0:
                    L.sh_gu = L.sh_down = L.sh_gate = None
                    return
            S = cfg.shared_expert_ffn // W      # under TP: this rank's features
            gp, up = gs[0], us[0]
            if W > 1:
                gp = split_rows(gs[0], gs[1], gs[2], tr * S, (tr + 1) * S)
                up = split_rows(us[0], us[1], us[2], tr * S, (tr + 1) * S)
            L.sh_gu = QLinear(torch.cat([gp, up]), gs[1], 2 * S, H, dev)
            t, qt2, shape = get(b + "ffn_down_shexp.weight")
            if W > 1:
                t = split_cols(t, qt2, shape, tr * S, (tr + 1) * S)
            L.sh_down = QLinear(t, qt2, shape[0], S, dev)
            if cfg.shared_expert_gated:
                t, qt3, _ = get(b + "ffn_gate_inp_shexp.weight")
                L.sh_gate = QLinear(t, qt3, 1, H, dev, f32_as_f16=True)

    def _linears(self):
        for L in self.layers:
            if L.linear:
                yield from (L.w_in, L.w_z, L.w_out)
            else:
                yield from (L.wqkv, L.wo)
            if L.experts is None:
                yield from (L.wgu, L.wdown)
            elif L.sh_gu is not None:
                yield from (L.sh_gu, L.sh_down)
        if self.last:
            yield self.head

    def weight_bytes(self) -> int:
        n = sum(l.nbytes for l in self._linears())
        for L in self.layers:
            if L.experts is not None:
                n += L.experts.nbytes
        return n

    def max_gemm_rows(self) -> int:
        c = self.cfg
        r = max(c.q_dim * (2 if c.attn_output_gate else 1) + 2 * c.kv_dim, 2 * c.ffn, c.hidden,
                2 * c.shared_expert_ffn)
        if self.n_lin_layers:
            r = max(r, (2 * c.ssm_k_heads + c.ssm_v_heads) * c.ssm_head_dim)
        return r

    def enable_lora(self, max_adapters: int = 4, max_rank: int = 64):
        """Allocate adapter tables (before contexts / CUDA graphs are made)."""
        from .lora import LoraSet
        assert self.tp is None, "LoRA on tensor-parallel shards is not supported"
        self.lora = LoraSet(self, max_adapters, max_rank)
        return self.lora

    def _lora(self, j: int, group: str, x, g, ctx, b):
        """Add the per-row adapter deltas of target `group` to GEMM result g."""
        if self.lora is None or b.lora_ids is None:
            return g
        t = self.lora.tables.get((j, group))
        if t is None:
            return g
        A, B, S, _ = t
        T, rows = x.shape[0], B.shape[1]
        delta = ctx.lora_delta[: T * rows].view(T, rows)
        C().lora_delta(x, b.lora_ids, A, B, S, ctx.lora_u, delta)
        return C().gemm_with_add(g, delta)

    def _row_parallel(self, lin, x, ctx):
        if self.tp is None:
            return lin(x, ctx.gemm)
        return self.tp.row_parallel(lin, x, ctx.gemm.status, ctx.gemm.num_sms)

    def _residual_norm(self, g, h, bias, w, out, ctx, post_w=None):
        """h += g (+ bias); out = RMSNorm(h) * w (w None: no normalised output).
        `post_w`: the branch output is RMSNorm-ed with it before the add.
        Under TP g holds the owner-routed partials and the sum over ranks, the
        residual add and the all-gather of h happen in one fused kernel."""
        eps = self.cfg.rms_eps
        if self.tp is not None:
            self.tp.reduce_norm(g, bias, w, out, eps, ctx.gemm.status, ctx.gemm.num_sms)
        else:
            C().epi_residual_rmsnorm(g, h, bias, w if w is not None else ctx.dummy_norm, out, eps,
                                     post_w)

    def _deltanet(self, L, b, kv, ctx, x, N):
        """Gated DeltaNet token mixing of one layer -> ctx.ssm_out (fp16)."""
        cfg = self.cfg
        nk, nv, dh = self.nk_loc, self.nv_loc, cfg.ssm_head_dim
        S = b.ssm_seqs.shape[0]
        g = L.w_in(x, ctx.gemm)
        C().ssm_conv_silu(g, L.conv_w, kv.conv_state(L.lin_idx), b.ssm_seqs, S, ctx.ssm_qkv[:N])
        gba = L.w_ba(x, ctx.gemm_side)
        gz = L.w_z(x, ctx.gemm)  # the conv consumed the in-projection's workspace already
        if b.ssm_max_rows > 32:  # prefill: chunked evaluation
            C().delta_chunk(ctx.ssm_qkv[:N], nk, nv, dh, gba, L.dt_bias, L.A, gz, L.ssm_norm,
                            cfg.rms_eps, kv.ssm_state(L.lin_idx), b.ssm_seqs, S,
                            ctx.ssm_oraw[:N], ctx.ssm_out[:N])
        else:
            C().delta_rule(ctx.ssm_qkv[:N], nk, nv, dh, gba, L.dt_bias, L.A, gz, L.ssm_norm,
                           cfg.rms_eps, kv.ssm_state(L.lin_idx), b.ssm_seqs, S, ctx.ssm_out[:N])

    def decode_launches(self) -> int:
        """Kernels of this stage's decode forward (what a captured graph replays)."""
        n = 2 if self.first else 1  # embed + rmsnorm (or the residual copy)
        for L in self.layers:
            if L.linear:
                n += 7   # in GEMM, conv, ba GEMM, z GEMM, delta rule, out GEMM, residual+norm
            else:
                n += 6 + (1 if L.gated else 0)  # qkv GEMM, rope/KV, attention + combine, o GEMM, residual+norm
            if L.experts is not None:
                # router GEMM + top-k, then plan/scatter/2 grouped GEMMs/combine, or under
                # expert parallelism send-counts/dispatch/wait/plan/2 GEMMs/wait/combine
                # (tensor parallelism: localize/plan/scatter/2 GEMMs/partial store/reduce)
                n += 2 + (8 if self.ep is not None else 7 if self.tp is not None else 5) + \
                    (3 + (L.sh_gate is not None) if L.sh_gu is not None else 0)
            else:
                n += 4   # gate|up GEMM, SwiGLU, down GEMM, residual+norm
        if self.last:
            n += 3       # head GEMM, logits copy, argmax (the row gather is a torch op)
        return n

    def make_context(self, max_tokens: int, max_samples: int, max_len: int):
        return GpuForwardContext(self, max_tokens, max_samples, max_len)

    def forward(self, b: StepBatch, kv: PagedKVCache, ctx: "GpuForwardContext",
                h_in: torch.Tensor | None = None) -> torch.Tensor:
        cfg = self.cfg
        N = b.tokens.shape[0]
        H, nq, nkv, d = cfg.hidden, self.n_q, self.n_kv, cfg.head_dim
        if self.tp is not None:
            self.tp.begin_forward()
        h = ctx.h[:N]
        if self.first:
            C().embed_gather(self.embd, self.embd_type, H, b.tokens, h)
            if cfg.embed_scale:
                h.mul_(cfg.embed_scale)
            if b.embed_rows is not None:  # image rows spliced into the prompt
                h.index_copy_(0, b.embed_rows.long(), b.embed_vals.to(h.dtype))
        elif h_in is not None and h_in.data_ptr() != h.data_ptr():
            h.copy_(h_in)
        x = ctx.x[:N]
        C().rmsnorm(h, self.layers[0].attn_norm, x, cfg.rms_eps)
        q = ctx.q[:N]
        ao = ctx.attn_out[:N]
        act = ctx.act[:N]
        P = self._stage_ctx()
        lev = getattr(self, "layer_events", None)   # per-layer CUDA events (layout planner)
        for j, L in enumerate(self.layers):
            if lev is not None:
                lev[j].record()
            if L.linear:
                with P("delta_rule"):
                    self._deltanet(L, b, kv, ctx, x, N)
                with P("o_proj+norm"):
                    g = self._row_parallel(L.w_out, ctx.ssm_out[:N], ctx)
                    self._residual_norm(g, h, None, L.ffn_norm, x, ctx)
            else:
                li = self.kv_off + L.kv_idx
                with P("qkv_proj+rope+kv_append"):
                    g = self._lora(j, "qkv", x, L.wqkv(x, ctx.gemm), ctx, b)
                    gate = ctx.gate[:N] if L.gated else None
                    inv, af = ((self.inv_freq_local, self.attn_factor_local) if L.local_rope
                               else (self.inv_freq, self.attn_factor))
                    C().epi_rope_kv(g, L.qkv_bias, b.positions, b.slots, inv, nq, nkv, d,
                                    cfg.rot_dim, cfg.rope_neox, af, q, kv.k(li),
                                    kv.v(li), kv.page_size, L.q_norm, L.k_norm, cfg.rms_eps, gate)
                with P("attention"):
                    paged_attention(q, kv.k(li), kv.v(li), b.block_table, b.seq_lens, ctx.attn,
                                    ao.view(N, nq, d), b.max_len, self.scale, L.window, L.sinks,
                                    softcap=cfg.attn_softcap,
                                    tree_mask=b.tree_mask, tree_start=b.tree_start,
                                    num_sms=ctx.gemm.num_sms, groups=b.groups)
                    if gate is not None:
                        C().mul_f16(ao, gate)
                with P("o_proj+norm"):
                    g = self._lora(j, "o", ao, self._row_parallel(L.wo, ao, ctx), ctx, b)
                    self._residual_norm(g, h, L.o_bias, L.ffn_norm, x, ctx, L.post_attn_norm)
            if j + 1 < len(self.layers):
                nxt_w, nxt_out = self.layers[j + 1].attn_norm, x
            elif self.last:
                nxt_w, nxt_out = self.out_norm, x
            else:
                nxt_w, nxt_out = None, None
            if L.experts is not None:
                with P("moe"):
                    # router logits live in the side workspace only until top-k
                    moe_route(x, L.router, L.router_b, ctx.moe, ctx.gemm_side,
                              mode=cfg.moe_mode, sel_b=L.sel_b, norm=cfg.moe_norm_topk,
                              scale=cfg.moe_scale)
                    sh = shg = None
                    if L.sh_gu is not None:
                        S = L.sh_gu.rows // 2
                        g = L.sh_gu(x, ctx.gemm)
                        C().epi_swiglu(g, None, S, 0, False, 0.0, 0.0, ctx.act_sh[:N])
                        shg = L.sh_gate(x, ctx.gemm_side) if L.sh_gate is not None else None
                        sh = L.sh_down(ctx.act_sh[:N], ctx.gemm)
                    if self.tp is not None:
                        g = moe_experts_tp(x, L.experts, ctx.moe, self.tp, sh, shg)
                        self._residual_norm(g, h, None, nxt_w, nxt_out, ctx)
                    elif self.ep is not None:
                        moe_experts_ep(x, L.experts, ctx.moe, self.ep, h, nxt_w, nxt_out, cfg.rms_eps,
                                       sh, shg)
                    else:
                        moe_experts(x, L.experts, ctx.moe, h, nxt_w, nxt_out, cfg.rms_eps, sh, shg)
                continue
            with P("ffn_gate_up+act"):
                g = self._lora(j, "gu", x, L.wgu(x, ctx.gemm), ctx, b)
                C().epi_swiglu(g, None, self.ffn_loc, self.act_kind, False, 0.0, 0.0, act)
            with P("ffn_down+norm"):
                g = self._lora(j, "down", act, self._row_parallel(L.wdown, act, ctx), ctx, b)
                self._residual_norm(g, h, None, nxt_w, nxt_out, ctx, L.post_ffn_norm)
        if lev is not None:
            lev[len(self.layers)].record()
        if not self.last:
            return h
        with P("lm_head"):
            S = b.sample_rows.shape[0]
            xs = ctx.xs[:S]
            torch.index_select(x, 0, b.sample_rows, out=xs)
            g = self.head(xs, ctx.gemm)
            logits = ctx.logits[:S]
            C().epi_copy(g, None, logits)
            if cfg.final_softcap:  # c * tanh(logits / c)
                logits.div_(cfg.final_softcap).tanh_().mul_(cfg.final_softcap)
            if cfg.logit_scale:  # granite: logits divided by its multiplier
                logits.div_(cfg.logit_scale)
        return logits

    def _stage_ctx(self):
        """Stage context of the profiler (SWARMLLM_PROFILE=1), outside CUDA-graph
        capture only; otherwise a no-op."""
        prof = getattr(self, "profiler", None)
        if prof is None or not prof.enabled or torch.cuda.is_current_stream_capturing():
            return _NO_STAGE
        return prof.stage


class _NullStage:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


_NULL_STAGE = _NullStage()


def _NO_STAGE(name: str):
    return _NULL_STAGE


class GpuForwardContext:
    """Preallocated activations and scratch for one model instance."""

    def __init__(self, model: LlamaGPU, max_tokens: int, max_samples: int, max_len: int):
        cfg, dev = model.cfg, model.device
        self.max_tokens, self.max_samples = max_tokens, max_samples
        head = ((max_samples, cfg.vocab),) if model.last else ()
        self.gemm = GemmWorkspace(dev, max_tokens, model.max_gemm_rows(), extra=head)
        # small side GEMMs whose results must outlive a main GEMM issued after
        # them (router logits, shared-expert gate, DeltaNet beta/decay)
        side_rows = max(cfg.n_experts, 2 * cfg.ssm_v_heads, 1)
        self.gemm_side = GemmWorkspace(dev, max_tokens, side_rows, self.gemm.num_sms)
        self.attn = AttentionWorkspace(dev, max_tokens, model.n_q, model.n_kv, cfg.head_dim,
                                       max_len, self.gemm.num_sms)
        H = cfg.hidden
        if model.tp is not None:
            # receive buffers for the row-parallel (hidden-wide) GEMMs; the residual
            # stream lives in the TP arena, where peers store their slices of it
            from ..ops.linear import stream_k_floats
            model.tp.setup(stream_k_floats(max_tokens, cfg.hidden, self.gemm.num_sms), max_tokens, H)
            self.h = model.tp.h_view()
            self.h.zero_()
        else:
            self.h = torch.zeros(max_tokens, H, dtype=torch.float32, device=dev)
        self.x = torch.zeros(max_tokens, H, dtype=torch.float16, device=dev)
        self.q = torch.zeros(max_tokens, model.n_q, cfg.head_dim, dtype=torch.float16, device=dev)
        self.attn_out = torch.zeros(max_tokens, model.n_q * cfg.head_dim, dtype=torch.float16,
                                    device=dev)
        self.act = torch.zeros(max_tokens, model.ffn_loc, dtype=torch.float16, device=dev)
        self.xs = torch.zeros(max_samples, H, dtype=torch.float16, device=dev)
        self.logits = torch.zeros(max_samples, cfg.vocab, dtype=torch.float32, device=dev)
        self.dummy_norm = torch.ones(H, dtype=torch.float32, device=dev)
        if cfg.attn_output_gate:
            self.gate = torch.zeros(max_tokens, model.n_q * cfg.head_dim, dtype=torch.float16,
                                    device=dev)
        if model.n_lin_layers:
            nk, nv, dh = model.nk_loc, model.nv_loc, cfg.ssm_head_dim
            self.ssm_qkv = torch.zeros(max_tokens, (2 * nk + nv) * dh, dtype=torch.float32,
                                       device=dev)
            self.ssm_out = torch.zeros(max_tokens, nv * dh, dtype=torch.float16, device=dev)
            self.ssm_oraw = torch.zeros(max_tokens, nv * dh, dtype=torch.float32, device=dev)
        if model.lora is not None:
            rows = max(t[1].shape[1] for t in model.lora.tables.values())
            R = max(t[0].shape[1] for t in model.lora.tables.values())
            self.lora_delta = torch.zeros(max_tokens * rows, dtype=torch.float32, device=dev)
            self.lora_u = torch.zeros(max_tokens * R, dtype=torch.float32, device=dev)
        self.moe = None
        exs = [L.experts for L in model.layers if L.experts is not None]
        if exs:
            ex = exs[0]
            self.moe = MoeWorkspace(dev, max_tokens, H, cfg.expert_ffn, cfg.n_experts,
                                    cfg.n_experts_used, ex.x_dtype, self.gemm.num_sms,
                                    ep=model.ep)
            # this rank's shared-expert features (the whole expert, or its TP share)
            S = max([L.sh_gu.rows // 2 for L in model.layers if L.sh_gu is not None] + [1])
            self.act_sh = torch.zeros(max_tokens, S, dtype=torch.float16, device=dev)
        # Size the CUDA-core GEMM scratch up front (graph capture cannot grow it).
        self.gemm.dense(max(max_tokens * model.max_gemm_rows(),
                            max_samples * cfg.vocab if model.last else 0) if _has_simt(model) else 0)


def _has_simt(model: LlamaGPU) -> bool:
    return any(not l.use_tc for l in model._linears())


# =========================================================================== CPU
class _QWeight:
    """Rows of a GGUF-quantized weight kept in their blocks, multiplied by the
    native CPU kernel (int8 activations, csrc/native/cpu_qmatmul.cpp)."""

    __slots__ = ("blocks", "qtype", "rows", "K", "expert_rows")
    FORMATS = (Q.Q4_K, Q.Q6_K, Q.Q8_0, Q.Q4_0, Q.IQ4_NL, Q.IQ4_XS, Q.MXFP4)
    SMALL = (Q.Q8_0, Q.Q4_0, Q.IQ4_NL, Q.MXFP4)      # 32-value blocks: any K % 32

    def __init__(self, blocks, qtype: int, rows: int, K: int):
        self.blocks = np.ascontiguousarray(blocks.reshape(rows, -1))
        self.qtype, self.rows, self.K = qtype, rows, K
        self.expert_rows = 0

    def __getitem__(self, sl: slice) -> "_QWeight":
        part = self.blocks[sl]
        return _QWeight(part, self.qtype, part.shape[0], self.K)

    @property
    def shape(self):
        return (self.rows, self.K)

    # from this many rows on (prefill), rows of the weight are dequantized a
    # slab at a time and multiplied in fp32: the int8 dot kernel's per-block
    # scale work grows with the rows, a GEMM's does not
    PREFILL_T = 192   # measured crossover on 8 AVX-512 cores: 4.5 vs 12 ms at 64 rows, 55 vs 22 at 512
    SLAB_FLOATS = 1 << 22

    def mm(self, x: torch.Tensor) -> torch.Tensor:
        from .. import _native
        x2 = x.reshape(-1, self.K).to(torch.float32).contiguous()
        T = x2.shape[0]
        if T >= self.PREFILL_T:
            out = torch.empty(T, self.rows, dtype=torch.float32)
            step = max(1, self.SLAB_FLOATS // self.K)
            for r0 in range(0, self.rows, step):
                n = min(step, self.rows - r0)
                w = torch.from_numpy(_native.cpu_dequant(self.blocks[r0:r0 + n], self.qtype, n,
                                                         self.K))
                torch.matmul(x2, w.T, out=out[:, r0:r0 + n])
            return out.reshape(*x.shape[:-1], self.rows).to(x.dtype)
        out = _native.cpu_qmatmul(self.blocks, self.qtype, self.rows, self.K, x2.numpy())
        return torch.from_numpy(out).reshape(*x.shape[:-1], self.rows).to(x.dtype)


class LlamaCPU:
    """fp32 PyTorch implementation on the host: the oracle for the GPU path and
    the engine backend for CPU-only runs (the two-CPU-peer tiny Llama).

    native=True is the optimised CPU inference path: dense Q4_K / Q6_K / Q8_0
    projections stay in their GGUF blocks and run through the native int8-dot
    matmul, attention through the native paged kernel (256-key chunks, online
    softmax) and the SwiGLU tail through the native vector exp; everything else
    (norms, RoPE, MoE routing, DeltaNet) keeps the fp32 PyTorch code.  The
    reference's CPU kernels are src/inference/split/attn_rows.rs,
    prefill_attn.rs and fast_math.rs."""

    def __init__(self, cfg: ModelConfig, source, layer_range: tuple[int, int] | None = None,
                 kv_layer_offset: int | None = None, dtype=torch.float32, native: bool = False,
                 mtp: bool = False):
        """mtp: also load the file's next-token-prediction block (the last
        stage of a model with `mtp_layers`), for `mtp_forward`."""
        self.cfg = cfg
        lo, hi = layer_range or (0, cfg.n_layers)
        self.lo, self.hi = lo, hi
        self.first, self.last = lo == 0, hi == cfg.n_layers
        # KV caches are stage-local: layer lo of this stage is cache layer 0.
        self.kv_off = 0 if kv_layer_offset is None else kv_layer_offset
        self.dtype = dtype
        self.native = bool(native) and dtype == torch.float32
        self._source = source
        self.nk_loc, self.nv_loc = cfg.ssm_k_heads, cfg.ssm_v_heads

        def dq(name):
            t, qt, shape = source.get(name)
            return torch.from_numpy(Q.dequantize(t.numpy().reshape(-1), qt).reshape(shape)).to(dtype)

        def lw(name):
            """A dense projection: kept quantized for the native path when its
            format and width allow, else dequantized."""
            if not self.native:
                return dq(name)
            t, qt, shape = source.get(name)
            width = 32 if qt in _QWeight.SMALL else 256
            if qt in _QWeight.FORMATS and len(shape) == 2 and shape[1] % width == 0:
                return _QWeight(t.numpy().reshape(-1), qt, shape[0], shape[1])
            return torch.from_numpy(Q.dequantize(t.numpy().reshape(-1), qt).reshape(shape)).to(dtype)

        if self.first:
            self.embd = dq("token_embd.weight")
        self.layers = []
        n_attn = n_lin = 0
        for i in range(lo, hi):
            b = f"blk.{i}."
            L = _GpuLayer()
            L.attn_norm, L.ffn_norm = dq(b + "attn_norm.weight"), dq(b + "ffn_norm.weight")
            L.linear = cfg.is_linear_attn(i)
            if L.linear:
                L.lin_idx = n_lin
                n_lin += 1
                L.w_in, L.w_z, L.w_ba = dq(b + "attn_qkv.weight"), dq(b + "attn_gate.weight"), dq(b + "ssm_ba.weight")
                L.conv_w, L.dt_bias, L.A = dq(b + "ssm_conv1d.weight"), dq(b + "ssm_dt.bias"), dq(b + "ssm_a")
                L.ssm_norm, L.w_out = dq(b + "ssm_norm.weight"), dq(b + "ssm_out.weight")
                self._load_ffn_cpu(L, b, dq, lw)
                self.layers.append(L)
                continue
            L.kv_idx = n_attn
            n_attn += 1
            self._load_attn(L, i, b, dq, lw)
            self._load_ffn_cpu(L, b, dq, lw)
            self.layers.append(L)
        self.n_kv_layers, self.n_lin_layers = n_attn, n_lin
        if self.last:
            self.out_norm = dq("output_norm.weight")
            self.head = lw("token_embd.weight" if cfg.tie_embeddings else "output.weight")
        self.mtp = None
        if mtp and cfg.mtp_layers and self.last:
            if not self.first:
                raise ValueError("the next-token-prediction block needs the token table")
            i = cfg.n_layers
            b = f"blk.{i}."
            M = _GpuLayer()
            M.attn_norm, M.ffn_norm = dq(b + "attn_norm.weight"), dq(b + "ffn_norm.weight")
            M.linear = False
            self._load_attn(M, i, b, dq, lw)
            self._load_ffn_cpu(M, b, dq, lw)
            M.eh_proj = lw(b + "nextn.eh_proj.weight")
            M.enorm, M.hnorm = dq(b + "nextn.enorm.weight"), dq(b + "nextn.hnorm.weight")
            hn = b + "nextn.shared_head_norm.weight"
            M.head_norm = dq(hn) if source.has(hn) else self.out_norm
            self.mtp = M
        inv, self.attn_factor = rope_inv_freq(cfg)
        self.inv_freq = torch.from_numpy(inv)
        inv_l, self.attn_factor_local = rope_inv_freq(cfg, local=True)
        self.inv_freq_local = torch.from_numpy(inv_l)
        self.scale = cfg.softmax_scale

    linear_state_spec = LlamaGPU.linear_state_spec

    def _load_attn(self, L, i, b, dq, lw):
        """A full-attention layer's weights (projections, biases, norms, sinks)."""
        cfg = self.cfg
        qr = cfg.q_dim * (2 if cfg.attn_output_gate else 1)
        if cfg.fused_qkv:
            wqkv = lw(b + "attn_qkv.weight")
            L.wq, L.wk, L.wv = wqkv[:qr], wqkv[qr:qr + cfg.kv_dim], wqkv[qr + cfg.kv_dim:]
            if cfg.attn_bias:
                bqkv = dq(b + "attn_qkv.bias")
                L.bq, L.bk, L.bv = bqkv[:qr], bqkv[qr:qr + cfg.kv_dim], bqkv[qr + cfg.kv_dim:]
            else:
                L.bq = L.bk = L.bv = None
        else:
            L.wq, L.wk, L.wv = lw(b + "attn_q.weight"), lw(b + "attn_k.weight"), lw(b + "attn_v.weight")
            L.bq = dq(b + "attn_q.bias") if cfg.attn_bias else None
            L.bk = dq(b + "attn_k.bias") if cfg.attn_bias else None
            L.bv = dq(b + "attn_v.bias") if cfg.attn_bias else None
        L.wo = lw(b + "attn_output.weight")
        L.bo = dq(b + "attn_output.bias") if cfg.has_out_bias else None
        L.post_attn = dq(b + "post_attention_norm.weight") if cfg.post_norms else None
        L.post_ffn = dq(b + "post_ffw_norm.weight") if cfg.post_norms else None
        L.local_rope = bool(cfg.rope_local_theta) and cfg.is_swa(i)
        L.q_norm = dq(b + "attn_q_norm.weight") if cfg.qk_norm else None
        L.k_norm = dq(b + "attn_k_norm.weight") if cfg.qk_norm else None
        L.sinks = dq(b + "attn_sinks.weight") if cfg.attn_sinks else None
        L.window = cfg.sliding_window if cfg.is_swa(i) else 0

    def _load_ffn_cpu(self, L, b, dq, lw=None):
        cfg = self.cfg
        lw = lw or dq
        L.moe = cfg.is_moe_layer(int(b.split(".")[1]))
        if L.moe:
            gpt = cfg.arch == "gpt-oss"
            L.wr = dq(b + "ffn_gate_inp.weight")
            L.br = dq(b + "ffn_gate_inp.bias") if gpt else None
            L.eg, L.eu, L.ed = (self._experts(b + n, dq) for n in (
                "ffn_gate_exps.weight", "ffn_up_exps.weight", "ffn_down_exps.weight"))
            L.ebg = dq(b + "ffn_gate_exps.bias") if gpt else None
            L.ebu = dq(b + "ffn_up_exps.bias") if gpt else None
            L.ebd = dq(b + "ffn_down_exps.bias") if gpt else None
            L.sel_b = (dq(b + "exp_probs_b.bias") if cfg.moe_gating == "sigmoid" and cfg.moe_sel_bias
                       else None)
            L.sg = L.sgi = None
            if cfg.shared_expert_ffn:
                L.sg, L.su, L.sd = (lw(b + n) for n in ("ffn_gate_shexp.weight", "ffn_up_shexp.weight",
                                                         "ffn_down_shexp.weight"))
                if cfg.shared_expert_gated:
                    L.sgi = dq(b + "ffn_gate_inp_shexp.weight")
        elif cfg.fused_gate_up:
            gu = lw(b + "ffn_up.weight")
            L.wg, L.wu, L.wd = gu[:cfg.ffn], gu[cfg.ffn:], lw(b + "ffn_down.weight")
        else:
            L.wg, L.wu, L.wd = lw(b + "ffn_gate.weight"), lw(b + "ffn_up.weight"), lw(b + "ffn_down.weight")

    def _experts(self, name, dq):
        """An expert stack [E, rows, K]: in native mode and a native format, one
        quantized [E * rows, K] matrix (expert e = its rows e*rows..), else the
        dequantized tensor."""
        if self.native:
            t, qt, shape = self._source.get(name)
            E, R, K = shape
            width = 32 if qt in _QWeight.SMALL else 256
            if qt in _QWeight.FORMATS and K % width == 0:
                W = _QWeight(t.numpy().reshape(-1), qt, E * R, K)
                W.expert_rows = R
                return W
        return dq(name)

    @staticmethod
    def _expert(W, e):
        """Expert e's [rows, K] weight of a stack from `_experts`."""
        if isinstance(W, _QWeight):
            R = W.expert_rows
            return W[e * R:(e + 1) * R]
        return W[e]

    @staticmethod
    def _mm(x, W):
        """x @ W.T for a dense tensor or a quantized weight (native path)."""
        return W.mm(x) if isinstance(W, _QWeight) else x @ W.T

    def _gate_act(self, g):
        if self.cfg.act == "gelu":
            return torch.nn.functional.gelu(g, approximate="tanh")
        return torch.nn.functional.silu(g)

    def _norm(self, x, w):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.cfg.rms_eps) * w

    def _rope(self, x, pos, local: bool = False):
        """x [N, heads, d] -> rotated (GGML norm pairs or NEOX halves, partial)."""
        cfg = self.cfg
        rd = cfg.rot_dim
        inv, af = (self.inv_freq_local, self.attn_factor_local) if local else (self.inv_freq,
                                                                             self.attn_factor)
        ang = pos.to(torch.float32)[:, None] * inv[None, :]
        c = (torch.cos(ang) * af)[:, None, :].to(x.dtype)
        s = (torch.sin(ang) * af)[:, None, :].to(x.dtype)
        out = x.clone()
        if cfg.rope_neox:
            a, b = x[..., : rd // 2], x[..., rd // 2: rd]
            out[..., : rd // 2] = a * c - b * s
            out[..., rd // 2: rd] = b * c + a * s
        else:
            a, b = x[..., 0:rd:2], x[..., 1:rd:2]
            out[..., 0:rd:2] = a * c - b * s
            out[..., 1:rd:2] = b * c + a * s
        return out

    def _lora_cpu(self, layer: int, suffix: str, x, y, b):
        """y += scale * B (A x) for the rows that carry an adapter using this weight."""
        ads = getattr(self, "lora_adapters", None)
        if not ads or b.lora_ids is None:
            return y
        base = f"blk.{layer}.{suffix}.weight"
        ids = b.lora_ids.long()
        for a, ad in enumerate(ads):
            if ad is None or base not in ad.tensors:   # a freed slot
                continue
            rows = (ids == a).nonzero().flatten()
            if len(rows) == 0:
                continue
            A_, B_ = (torch.from_numpy(t).to(y.dtype) for t in ad.tensors[base])
            y = y.clone()
            y[rows] += ad.scale(base) * ((x[rows] @ A_.T) @ B_.T)
        return y

    def _act(self, g, u):
        cfg = self.cfg
        if not cfg.swiglu_limit:
            return torch.nn.functional.silu(g) * u
        g = torch.clamp(g, max=cfg.swiglu_limit)
        u = torch.clamp(u, -cfg.swiglu_limit, cfg.swiglu_limit)
        return g * torch.sigmoid(cfg.swiglu_alpha * g) * (u + 1)

    def _glu(self, g, u):
        if self.native and self.cfg.act != "gelu":
            from .. import _native
            return torch.from_numpy(_native.cpu_silu_mul(g.contiguous().numpy(),
                                                         u.contiguous().numpy()))
        return self._gate_act(g) * u

    def _ffn(self, L, x, layer: int = -1, b=None):
        if L.moe:
            return self._moe(x, L)
        mm = self._mm
        if b is None:
            return mm(self._glu(mm(x, L.wg), mm(x, L.wu)), L.wd)
        gg = self._lora_cpu(layer, "ffn_gate", x, mm(x, L.wg), b)
        uu = self._lora_cpu(layer, "ffn_up", x, mm(x, L.wu), b)
        act = self._glu(gg, uu)
        return self._lora_cpu(layer, "ffn_down", act, mm(act, L.wd), b)

    def _deltanet(self, L, x, b, kv):
        """Gated DeltaNet (sequential recurrence, the definition the GPU
        kernels implement): conv1d + SiLU, L2-normalised q/k, decay and beta
        gates, delta-rule state update, gated RMSNorm, out-projection."""
        cfg = self.cfg
        nk, nv, D = cfg.ssm_k_heads, cfg.ssm_v_heads, cfg.ssm_head_dim
        K = cfg.ssm_conv_kernel
        rep = nv // nk
        N = x.shape[0]
        qkv, z, ba = x @ L.w_in.T, x @ L.w_z.T, x @ L.w_ba.T
        conv_st, ssm_st = kv.conv_state(L.lin_idx), kv.ssm_state(L.lin_idx)
        out = torch.zeros(N, nv * D, dtype=x.dtype)
        for r0, n, slot, p0 in b.ssm_seqs.tolist():
            if n <= 0:
                continue
            win = torch.zeros(K - 1, qkv.shape[1], dtype=x.dtype) if p0 == 0 else conv_st[slot].to(x.dtype)
            xs = torch.cat([win, qkv[r0:r0 + n]], 0)
            act = sum(L.conv_w[:, i] * xs[i:i + n] for i in range(K))
            act = torch.nn.functional.silu(act)
            conv_st[slot] = xs[-(K - 1):].to(conv_st.dtype)
            S = torch.zeros(nv, D, D, dtype=x.dtype) if p0 == 0 else ssm_st[slot].to(x.dtype)
            if self.native:
                out[r0:r0 + n] = self._deltanet_native(L, act, ba[r0:r0 + n], z[r0:r0 + n], S)
                ssm_st[slot] = S.to(ssm_st.dtype)
                continue
            for t in range(n):
                a = act[t]
                q = a[:nk * D].view(nk, D)
                k = a[nk * D:2 * nk * D].view(nk, D)
                v = a[2 * nk * D:].view(nv, D)
                q = q * torch.rsqrt(q.pow(2).sum(-1, keepdim=True) + 1e-6) / math.sqrt(D)
                k = k * torch.rsqrt(k.pow(2).sum(-1, keepdim=True) + 1e-6)
                q, k = q.repeat_interleave(rep, 0), k.repeat_interleave(rep, 0)
                r = r0 + t
                beta = torch.sigmoid(ba[r, :nv])
                g = L.A * torch.nn.functional.softplus(ba[r, nv:] + L.dt_bias)
                S = S * torch.exp(g)[:, None, None]
                kvm = torch.einsum("hij,hi->hj", S, k)
                dl = (v - kvm) * beta[:, None]
                S = S + k[:, :, None] * dl[:, None, :]
                o = torch.einsum("hij,hi->hj", S, q)
                o = o * torch.rsqrt(o.pow(2).mean(-1, keepdim=True) + cfg.rms_eps) * L.ssm_norm
                o = o * torch.nn.functional.silu(z[r].view(nv, D))
                out[r] = o.flatten()
            ssm_st[slot] = S.to(ssm_st.dtype)
        return out @ L.w_out.T

    def _deltanet_native(self, L, act, ba, z, S):
        """The same recurrence with the per-row gates and norms as whole-block
        torch ops and the state update in the native kernel (S in place)."""
        from .. import _native
        cfg = self.cfg
        nk, nv, D = cfg.ssm_k_heads, cfg.ssm_v_heads, cfg.ssm_head_dim
        n = act.shape[0]
        q = act[:, :nk * D].reshape(n, nk, D)
        k = act[:, nk * D:2 * nk * D].reshape(n, nk, D)
        v = act[:, 2 * nk * D:].reshape(n, nv, D)
        q = q * torch.rsqrt(q.pow(2).sum(-1, keepdim=True) + 1e-6) / math.sqrt(D)
        k = k * torch.rsqrt(k.pow(2).sum(-1, keepdim=True) + 1e-6)
        beta = torch.sigmoid(ba[:, :nv])
        g = L.A * torch.nn.functional.softplus(ba[:, nv:] + L.dt_bias)
        st = S.numpy()
        o = torch.from_numpy(_native.cpu_delta_rule(
            q.float().contiguous().numpy(), k.float().contiguous().numpy(),
            v.float().contiguous().numpy(), g.float().contiguous().numpy(),
            beta.float().contiguous().numpy(), st))
        o = o * torch.rsqrt(o.pow(2).mean(-1, keepdim=True) + cfg.rms_eps) * L.ssm_norm
        o = o * torch.nn.functional.silu(z.reshape(n, nv, D))
        return o.reshape(n, nv * D)

    def _moe(self, x, L):
        """Routed experts (top-k softmax) + optional sigmoid-gated shared expert
        (reference: MoeFfn, src/inference/layers/moe.rs)."""
        cfg = self.cfg
        k = cfg.n_experts_used
        logits = x @ L.wr.T + (L.br if L.br is not None else 0)
        if cfg.moe_gating == "sigmoid":
            # sigmoid scores; the selection bias picks the experts but does not weigh them
            score = torch.sigmoid(logits)
            sel = score + (L.sel_b if L.sel_b is not None else 0)
            top_i = torch.topk(sel, k, dim=-1).indices
            w = torch.gather(score, 1, top_i)
            if cfg.moe_norm_topk:
                w = w / w.sum(-1, keepdim=True)
            w = w * cfg.moe_scale
        else:
            top_v, top_i = torch.topk(logits, k, dim=-1)
            if cfg.moe_softmax_after_topk:
                w = torch.softmax(top_v, -1)
            else:
                w = torch.gather(torch.softmax(logits, -1), 1, top_i)
        y = torch.zeros_like(x)
        for e in top_i.unique().tolist():
            sel = top_i == e
            rows = sel.any(1).nonzero().flatten()
            we = (w * sel).sum(1)[rows]
            xs = x[rows]
            if cfg.moe_weight_input:  # llama4: the expert sees its weight times the input
                xs, we = xs * we[:, None], torch.ones_like(we)
            mm, ex = self._mm, self._expert
            g = mm(xs, ex(L.eg, e)) + (L.ebg[e] if L.ebg is not None else 0)
            u = mm(xs, ex(L.eu, e)) + (L.ebu[e] if L.ebu is not None else 0)
            o = mm(self._act(g, u), ex(L.ed, e)) + (L.ebd[e] if L.ebd is not None else 0)
            y[rows] += we[:, None] * o
        if L.sg is not None:
            gate = torch.sigmoid(x @ L.sgi)[:, None] if L.sgi is not None else 1.0
            y = y + gate * self._mm(self._glu(self._mm(x, L.sg), self._mm(x, L.su)), L.sd)
        return y

    def forward(self, b: StepBatch, kv: PagedKVCache, ctx=None, h_in=None,
                want_hidden: bool = False, capture=()) -> torch.Tensor:
        """Logits of the sample rows (the last stage), or the residual stream
        (other stages).  want_hidden: also the output-normed hidden state of
        every row, (logits, hidden) -- what a next-token-prediction head reads.
        capture: absolute layer indices whose INPUT residual stream (every row)
        is kept in self.captured[layer] (n_layers: the stream after the last
        layer) -- what a block drafter reads."""
        cfg = self.cfg
        self.captured = {}
        h = self.embd[b.tokens.long()].clone() if self.first else h_in.to(self.dtype).clone()
        if self.first and cfg.embed_scale:
            h = h * cfg.embed_scale
        if self.first and b.embed_rows is not None:  # image rows spliced into the prompt
            h.index_copy_(0, b.embed_rows.long(), b.embed_vals.to(h.dtype))
        ps = kv.page_size
        slots = b.slots.long()
        pages, offs = slots // ps, slots % ps
        for j, L in enumerate(self.layers):
            if self.lo + j in capture:
                self.captured[self.lo + j] = h.clone()
            x = self._norm(h, L.attn_norm)
            if L.linear:
                h = h + self._deltanet(L, x, b, kv)
                x = self._norm(h, L.ffn_norm)
                h = h + self._ffn(L, x)
                continue
            h = self._attn_layer(L, self.lo + j, h, x, b, kv, self.kv_off + L.kv_idx, pages, offs)
        if self.hi in capture:
            self.captured[self.hi] = h.clone()
        if not self.last:
            return h
        x = self._norm(h[b.sample_rows.long()], self.out_norm)
        logits = self._logits(x)
        if want_hidden:
            return logits, self._norm(h, self.out_norm)
        return logits

    def mtp_forward(self, tokens: torch.Tensor, hidden: torch.Tensor, b: StepBatch,
                    kv: PagedKVCache):
        """The next-token-prediction block: row r pairs token tokens[r] (the
        token at position b.positions[r]) with `hidden[r]`, the output-normed
        trunk state at the position before it, and predicts the token after:
        eh_proj([enorm(embedding) | hnorm(hidden)]) -> one full-attention layer
        over its own one-layer cache `kv` -> head norm -> the output head.
        Returns (logits of b.sample_rows, head-normed state of every row, which
        the next draft step reads as its hidden state).  As llama.cpp's
        qwen35 graph_mtp / the reference's split/mtp.rs lay it out."""
        M = self.mtp
        e = self._norm(self.embd[tokens.long()].to(self.dtype), M.enorm)
        x_res = self._mm(torch.cat([e, self._norm(hidden.to(self.dtype), M.hnorm)], -1), M.eh_proj)
        ps = kv.page_size
        slots = b.slots.long()
        h = self._attn_layer(M, self.cfg.n_layers, x_res, self._norm(x_res, M.attn_norm), b, kv, 0,
                             slots // ps, slots % ps)
        out = self._norm(h, M.head_norm)
        return self._logits(out[b.sample_rows.long()]), out

    def _logits(self, x):
        logits = self._mm(x, self.head)
        if self.cfg.final_softcap:
            logits = self.cfg.final_softcap * torch.tanh(logits / self.cfg.final_softcap)
        if self.cfg.logit_scale:
            logits = logits / self.cfg.logit_scale
        return logits

    def _attn_layer(self, L, layer, h, x, b, kv, li, pages, offs):
        """One full-attention decoder layer: x = attn_norm(h) in, the new
        residual out (attention, output gate, post-norms, FFN)."""
        cfg = self.cfg
        N = x.shape[0]
        nq, nkv, d = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
        mm = self._mm
        q = self._lora_cpu(layer, "attn_q", x, mm(x, L.wq), b)
        k = self._lora_cpu(layer, "attn_k", x, mm(x, L.wk), b)
        v = self._lora_cpu(layer, "attn_v", x, mm(x, L.wv), b)
        gate = None
        if cfg.attn_output_gate:
            qg = q.view(N, nq, 2 * d)
            q, gate = qg[..., :d], torch.sigmoid(qg[..., d:]).reshape(N, nq * d)
        if L.bq is not None:
            q, k, v = q + L.bq, k + L.bk, v + L.bv
        q, k, v = q.reshape(N, nq, d), k.view(N, nkv, d), v.view(N, nkv, d)
        if L.q_norm is not None:
            q, k = self._norm(q, L.q_norm), self._norm(k, L.k_norm)
        if not cfg.is_nope(layer):
            if cfg.qk_rms_plain:
                # llama4 normalises after RoPE; a rotation keeps every pair's
                # length, so the head's RMS (and this result) is the same
                q, k = self._norm(q, 1.0), self._norm(k, 1.0)
            q, k = self._rope(q, b.positions, L.local_rope), self._rope(k, b.positions, L.local_rope)
        K, V = kv.k(li), kv.v(li)
        K[pages, :, offs, :] = k.to(K.dtype)
        V[pages, :, offs, :] = v.to(V.dtype)
        if self.native:
            att = self._attention_native(L, q, K, V, b)
        else:
            att = self._attention(L, q, K, V, b)
        a = att.view(N, nq * d)
        if gate is not None:
            a = a * gate
        o = self._lora_cpu(layer, "attn_output", a, mm(a, L.wo), b)
        if L.bo is not None:
            o = o + L.bo
        if L.post_attn is not None:
            o = self._norm(o, L.post_attn)
        rs = cfg.residual_scale or 1.0
        h = h + o * rs
        x = self._norm(h, L.ffn_norm)
        f = self._ffn(L, x, layer, b)
        if L.post_ffn is not None:
            f = self._norm(f, L.post_ffn)
        return h + f * rs

    def _attention(self, L, q, K, V, b):
        """The fp32 oracle: per row, gather its keys and take a plain softmax."""
        cfg = self.cfg
        N, nq, d = q.shape
        rep = nq // K.shape[1]
        ps = K.shape[2]
        att = torch.empty(N, nq, d, dtype=self.dtype)
        for t in range(N):
            Lt = int(b.seq_lens[t])
            lo = max(0, Lt - L.window) if L.window else 0
            keys = torch.arange(lo, Lt)
            bt = b.block_table[t].long()
            kp, ko = bt[keys // ps], keys % ps
            kk = K[kp, :, ko, :].to(self.dtype)  # [n, nkv, d]
            vv = V[kp, :, ko, :].to(self.dtype)
            vis = torch.ones(len(keys), dtype=torch.bool)
            if b.tree_mask is not None:
                ts = int(b.tree_start[t])
                m = int(b.tree_mask[t]) & ((1 << 64) - 1)
                rel = keys - ts
                vis = (rel < 0) | torch.tensor([(rr >= 0 and rr < 64 and (m >> int(rr)) & 1 == 1)
                                                for rr in rel.tolist()], dtype=torch.bool)
            kk = kk.repeat_interleave(rep, dim=1)
            vv = vv.repeat_interleave(rep, dim=1)
            s = torch.einsum("hd,nhd->hn", q[t], kk) * self.scale
            if cfg.attn_softcap:
                s = cfg.attn_softcap * torch.tanh(s / cfg.attn_softcap)
            s = s.masked_fill(~vis[None, :], float("-inf"))
            if L.sinks is not None:
                s = torch.cat([s, L.sinks[:, None]], 1)
            p = torch.softmax(s, -1)
            if L.sinks is not None:
                p = p[:, :-1]
            att[t] = torch.einsum("hn,nhd->hd", p, vv)
        return att

    def _attention_native(self, L, q, K, V, b):
        from .. import _native
        opt = {}
        if b.tree_mask is not None:
            opt["tree_start"] = b.tree_start.numpy()
            opt["tree_mask"] = b.tree_mask.numpy()
        if L.sinks is not None:
            opt["sinks"] = L.sinks.float().numpy()
        out = _native.cpu_paged_attention(
            q.to(torch.float32).contiguous().numpy(), K.numpy(), V.numpy(),
            b.block_table.numpy(), b.seq_lens.numpy(), float(self.scale), window=int(L.window),
            softcap=float(self.cfg.attn_softcap or 0.0), **opt)
        return torch.from_numpy(out).to(self.dtype)
