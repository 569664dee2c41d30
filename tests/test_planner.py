"""Layout planner (CPU): per-layer costs follow what a layer reads, stage cuts
balance unequal layers, the (pipeline x tensor-parallel) layout for a fixed
batch prefers tensor parallelism, memory rules out layouts that do not fit,
and TP groups follow peer access."""
from swarmllm_b200.models.config import preset
from swarmllm_b200.parallel.planner import (layer_costs, layer_weight_bytes, plan_layout,
                                            stage_plan, tp_groups)


def test_layer_costs_follow_bytes():
    cfg = preset("llama-3.3-70b")
    c1, c32 = layer_costs(cfg, 1, 2048), layer_costs(cfg, 32, 2048)
    assert len(c1) == 80 and all(b > a for a, b in zip(c1, c32))   # more KV at batch 32
    t2 = layer_costs(cfg, 32, 2048, tp=2)
    assert all(b < a for a, b in zip(c32, t2))                       # half the bytes per GPU
    read, whole = layer_weight_bytes(cfg, 0)
    assert read == whole and 4.5e8 < read < 5.2e8                    # ~0.48 GB of Q4_K per layer


def test_hybrid_stage_cuts_balance_unequal_layers():
    cfg = preset("qwen3-next-80b-a3b-style")
    costs = layer_costs(cfg, 8, 32768)
    lin = [c for l, c in enumerate(costs) if cfg.is_linear_attn(l)]
    full = [c for l, c in enumerate(costs[:-1]) if not cfg.is_linear_attn(l)]
    assert min(full) > max(lin)          # 32k of KV makes full-attention layers dearer
    b, worst = stage_plan(costs, [0.0] * len(costs), 4)
    loads = [sum(costs[b[s]:b[s + 1]]) for s in range(4)]
    assert abs(max(loads) - worst) < 1e-12 and max(loads) - min(loads) < max(costs)
    uniform = [0, 12, 24, 36, 48]
    assert max(sum(costs[uniform[s]:uniform[s + 1]]) for s in range(4)) >= worst


def test_fixed_batch_prefers_tensor_parallel_and_memory_limits():
    cfg = preset("llama-3.3-70b")
    ls = plan_layout(cfg, 8, 32, 2304)
    assert ls[0].fits and ls[0].tp == 8 and ls[0].pp == 1
    by = {(l.pp, l.tp): l for l in ls}
    assert by[(4, 2)].step_s > by[(1, 8)].step_s
    # 70B does not fit on one 40 GB GPU; it does on one 180 GB GPU
    assert not plan_layout(cfg, 1, 32, 2304, gpu_mem=40e9)[0].fits
    assert plan_layout(cfg, 1, 32, 2304)[0].fits


def test_tp_groups_follow_peer_access():
    links = {(0, 1), (1, 0), (2, 3), (3, 2)}     # two NVLink islands
    g = tp_groups(4, lambda a, b: (a, b) in links)
    assert g == [[0, 1], [2, 3]]
    assert tp_groups(8, lambda a, b: True) == [list(range(8))]
