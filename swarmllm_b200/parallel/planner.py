"""Layout planning for one node: what each layer costs, how to cut the layers
into pipeline stages, how many GPUs to put in each tensor-parallel group.

The reference prices a chain of peers by measured per-layer latency, RTT and
load (chain_cost_terms / route_shortest_path, src/inference/scheduler/
parallax.rs:1040,1154) and groups LAN peers into tensor-parallel segments
(detect_tp_groups, src/inference/scheduler/mod.rs:7764).  Here the peers are
the GPUs of one NVSwitch box, so:

* ``layer_costs`` prices every layer of a model for a decode step from what it
  must read (its weights, the KV of the batch, recurrent state, the experts the
  batch routes to) at the measured HBM bandwidth, plus the fused TP reduce's
  latency per row-parallel layer; ``measured_layer_costs`` replaces the
  estimate by CUDA-event timings of the model's own layers on the device.
* ``stage_plan`` cuts the layers with the native bottleneck DP
  (csrc/native/planner.cpp) under per-GPU memory capacity.
* ``tp_groups`` finds the GPUs that reach each other's memory (peer access:
  the same NVSwitch fabric), the candidates for one TP group.
* ``plan_layout`` tries every (pipeline stages x TP group size) split of N
  GPUs that fits in memory and keeps the fastest predicted decode step for a
  global batch; with V = stages waves the pipeline reads each stage's weights
  once per wave, so a fixed batch gains from TP, a growing batch from PP.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

from ..gguf import quants as Q
from ..models.config import ModelConfig
from ..utils.ext import native

HBM_GBS = 6538.0          # measured copy bandwidth of one B200 (GB/s)
TP_REDUCE_US = 10.0       # fused reduce + all-gather latency per row-parallel layer
KERNEL_US = 3.0           # fixed cost of one kernel boundary in a captured step


def _qbytes(qtype: str, n: int) -> float:
    t = Q.NAME_TO_TYPE[qtype]
    bv, bb = Q.BLOCK[t]
    return n / bv * bb


def layer_weight_bytes(cfg: ModelConfig, layer: int) -> tuple[float, float]:
    """(bytes every step reads, bytes of the whole layer) for one layer."""
    H, wq = cfg.hidden, cfg.weight_qtype
    if cfg.is_linear_attn(layer):
        nk, nv, dh = cfg.ssm_k_heads, cfg.ssm_v_heads, cfg.ssm_head_dim
        mix = _qbytes(wq, H * (2 * nk * dh + nv * dh)) + _qbytes(wq, H * nv * dh) * 2
    else:
        q = cfg.q_dim * (2 if cfg.attn_output_gate else 1)
        mix = _qbytes(wq, H * (q + 2 * cfg.kv_dim)) + _qbytes(wq, cfg.q_dim * H)
    if cfg.is_moe_layer(layer):
        xq = cfg.expert_qtype or wq
        per_expert = 3 * _qbytes(xq, H * cfg.expert_ffn)
        shared = 3 * _qbytes(wq, H * cfg.shared_expert_ffn) if cfg.shared_expert_ffn else 0.0
        return mix + shared, mix + shared + cfg.n_experts * per_expert
    ffn = 3 * _qbytes(wq, H * cfg.ffn)
    return mix + ffn, mix + ffn


def layer_costs(cfg: ModelConfig, batch: int, context: int, tp: int = 1,
                hbm_gbs: float = HBM_GBS) -> list[float]:
    """Seconds per layer of one decode step of `batch` sequences at `context`
    tokens, on one GPU of a `tp`-way group."""
    out = []
    for l in range(cfg.n_layers):
        read, _ = layer_weight_bytes(cfg, l)
        if cfg.is_moe_layer(l):  # the experts this batch routes to (uniform routing)
            used = cfg.n_experts * (1 - (1 - cfg.n_experts_used / cfg.n_experts) ** batch)
            xq = cfg.expert_qtype or cfg.weight_qtype
            read += used * 3 * _qbytes(xq, cfg.hidden * cfg.expert_ffn)
        if cfg.is_linear_attn(l):
            state = cfg.ssm_v_heads * cfg.ssm_head_dim * cfg.ssm_head_dim * 4 * 2
            read += batch * state
        else:
            span = min(context, cfg.sliding_window) if cfg.is_swa(l) else context
            read += batch * span * cfg.kv_dim * 2 * 2          # fp16 K and V pages
        t = read / tp / (hbm_gbs * 1e9)
        t += 8 * KERNEL_US * 1e-6                              # the layer's launches
        if tp > 1:
            t += 2 * TP_REDUCE_US * 1e-6
        out.append(t)
    if out:   # embedding gather / LM head on the first / last layer
        head = _qbytes(cfg.output_qtype or cfg.weight_qtype, cfg.vocab * cfg.hidden)
        out[-1] += head / (hbm_gbs * 1e9)
    return out


def measured_layer_costs(model, batch_fn, repeats: int = 3) -> list[float]:
    """Per-layer seconds of `model` (a LlamaGPU) measured on the device: CUDA
    events at every layer boundary of `repeats` forwards of batch_fn()'s
    (batch, kv, ctx)."""
    import torch
    n = len(model.layers)
    tot = [0.0] * n
    for _ in range(repeats + 1):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(n + 1)]
        model.layer_events = ev
        b, kv, ctx = batch_fn()
        model.forward(b, kv, ctx)
        torch.cuda.synchronize()
        if _ > 0:   # the first run warms up
            for i in range(n):
                tot[i] += ev[i].elapsed_time(ev[i + 1]) / 1e3
    model.layer_events = None
    return [t / repeats for t in tot]


@dataclass
class Layout:
    pp: int
    tp: int
    bounds: list
    step_s: float
    fits: bool

    @property
    def gpus(self) -> int:
        return self.pp * self.tp


def stage_plan(costs: list[float], layer_mem: list[float], n_stages: int,
               gpu_mem: float = 1e30) -> tuple[list[int], float]:
    """Layer boundaries [S+1] minimising the slowest stage under each GPU's
    memory (native DP); returns (boundaries, bottleneck seconds)."""
    plan = native().plan_bottleneck(list(map(float, costs)), list(map(float, layer_mem)),
                                    [1.0] * n_stages, [float(gpu_mem)] * n_stages, 0.0)
    if not plan.feasible:
        raise ValueError(f"cannot split {len(costs)} layers into {n_stages} stages")
    return list(plan.first_layer), float(plan.bottleneck)


def plan_layout(cfg: ModelConfig, n_gpus: int, batch: int, context: int,
                gpu_mem: float = 180e9, kv_bytes_per_token: float | None = None,
                hbm_gbs: float = HBM_GBS) -> list[Layout]:
    """Every (pp, tp) with pp * tp == n_gpus, best first by predicted decode
    step time at `batch` sequences (waves = pp), unfit ones last."""
    kvt = kv_bytes_per_token if kv_bytes_per_token is not None else \
        sum(cfg.kv_dim * 2 * 2 for l in range(cfg.n_layers) if not cfg.is_linear_attn(l))
    out = []
    for tp in (t for t in range(1, n_gpus + 1) if n_gpus % t == 0):
        pp = n_gpus // tp
        if cfg.n_heads % tp or cfg.n_kv_heads % tp or (cfg.hidden // 128) % tp or \
                cfg.ffn % (256 * tp) or pp > cfg.n_layers:
            continue
        waves = min(pp, batch)
        per_wave = max(1, math.ceil(batch / waves))
        costs = layer_costs(cfg, per_wave, context, tp, hbm_gbs)
        mem = [layer_weight_bytes(cfg, l)[1] / tp + batch * context * kvt / cfg.n_layers / tp
               for l in range(cfg.n_layers)]
        try:
            bounds, bottleneck = stage_plan(costs, mem, pp, gpu_mem)
            fits = True
        except ValueError:
            bounds, bottleneck, fits = [], float("inf"), False
        # every wave passes every stage once per step; stages work in parallel
        step = bottleneck * waves if fits else float("inf")
        out.append(Layout(pp, tp, bounds, step, fits))
    return sorted(out, key=lambda x: (not x.fits, x.step_s))


def tp_groups(n_gpus: int | None = None, can_access=None) -> list[list[int]]:
    """Groups of GPUs that can all reach each other's memory (peer access over
    NVLink / NVSwitch): each group may host one tensor-parallel segment."""
    if can_access is None:
        import torch
        n_gpus = torch.cuda.device_count() if n_gpus is None else n_gpus
        can_access = torch.cuda.can_device_access_peer
    groups: list[list[int]] = []
    for d in range(n_gpus):
        for g in groups:
            if all(can_access(d, o) and can_access(o, d) for o in g):
                g.append(d)
                break
        else:
            groups.append([d])
    return groups
