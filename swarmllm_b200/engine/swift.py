"""SWIFT-style self-speculation: the target model drafts for itself with a
contiguous block of its middle layers skipped, so no drafter weights are
needed; the full target verifies the draft tree as with any drafter.

The skipped block is `skip_ratio` of the layers, never the first two or the
last two (the outer layers shape the output distribution most).  Candidate
patterns differ in where the block starts; `skip_patterns` lists them and
`SkipCalibrator` keeps per-pattern acceptance counts and names the best one.
A drafter built on one pattern keeps its own KV cache of the layers it runs.

Reference behaviour: SWIFT (Xia et al. 2024, arXiv 2410.06916) as the
reference applies it: skip mask of a contiguous middle block with the outer
layers kept (src/inference/swift.rs:20,119), candidates varying the block's
start, the best acceptance pinned after a calibration window.
"""
from __future__ import annotations

import copy


def skip_patterns(n_layers: int, skip_ratio: float = 0.45, max_candidates: int = 5):
    """Candidate skip masks (True = skipped): a block of round(ratio * L)
    layers inside [2, L - 2), at up to `max_candidates` evenly spaced starts."""
    if n_layers < 5 or skip_ratio <= 0:
        return [[False] * n_layers]
    skip = min(round(n_layers * min(skip_ratio, 0.95)), n_layers - 4)
    if skip <= 0:
        return [[False] * n_layers]
    lo, hi = 2, n_layers - 2 - skip          # feasible block starts
    n = min(max_candidates, hi - lo + 1)
    starts = sorted({lo + round(i * (hi - lo) / max(n - 1, 1)) for i in range(n)})
    # the centred block first: the single pattern when no calibration runs
    mid = lo + (hi - lo) // 2
    starts = ([mid] + [s for s in starts if s != mid])[:max_candidates]
    return [[start <= l < start + skip for l in range(n_layers)] for start in starts]


class SkipCalibrator:
    """Acceptance per candidate pattern; best() is the highest rate seen."""

    def __init__(self, patterns):
        self.patterns = patterns
        self.accepted = [0] * len(patterns)
        self.drafted = [0] * len(patterns)

    def record(self, i: int, accepted: int, drafted: int):
        self.accepted[i] += accepted
        self.drafted[i] += drafted

    def best(self) -> int:
        rates = [a / d if d else -1.0 for a, d in zip(self.accepted, self.drafted)]
        return max(range(len(rates)), key=lambda i: rates[i])


def layer_skip_drafter(target, mask):
    """A view of `target` (a LlamaGPU) that runs only the layers the mask
    keeps.  Weights are shared; every layer keeps its KV / state index, so the
    drafter's own cache is laid out as the target's."""
    assert len(mask) == len(target.layers)
    d = copy.copy(target)
    d.layers = [L for L, skip in zip(target.layers, mask) if not skip]
    d.skipped = sum(mask)
    return d
