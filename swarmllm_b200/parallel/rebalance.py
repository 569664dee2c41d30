"""Stage rebalancing for the pipeline engines: measured per-stage step times
re-weight the layer cost model, and when a new cut would make the slowest
stage clearly faster, every rank rebuilds its stage with the new layer range
(the same rebuild the failover path does, without a failure).

Reference behaviour: the shard rebalancer moves layer ranges between peers
when their measured load diverges (src/health/rebalancer.rs:18); here the
"peers" are the GPUs of one node and the move is a re-cut of the layer
ranges followed by a reload of each rank's layers.
"""
from __future__ import annotations

from .planner import stage_plan


class StageRebalancer:
    def __init__(self, layer_costs: list[float], threshold: float = 0.1):
        """`layer_costs`: the model's per-layer cost estimate (planner.layer_costs
        or measured); `threshold`: the minimum relative gain of the slowest
        stage that justifies a rebuild."""
        self.costs = list(map(float, layer_costs))
        self.threshold = threshold

    def reweighted(self, bounds: list[int], stage_s: list[float]) -> list[float]:
        """Per-layer costs scaled so each stage's sum equals its measured time."""
        out = []
        for s in range(len(bounds) - 1):
            seg = self.costs[bounds[s]:bounds[s + 1]]
            pred = sum(seg) or 1.0
            f = stage_s[s] / pred
            out += [c * f for c in seg]
        return out

    def propose(self, bounds: list[int], stage_s: list[float]) -> list[int] | None:
        """New boundaries, or None if the cut is good enough."""
        costs = self.reweighted(bounds, stage_s)
        new, bottleneck = stage_plan(costs, [0.0] * len(costs), len(bounds) - 1)
        if new != list(bounds) and bottleneck < max(stage_s) * (1.0 - self.threshold):
            self.costs = costs          # measured weights carry into the next round
            return new
        return None
