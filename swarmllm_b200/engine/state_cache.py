"""Prefix cache for hybrid models: saved recurrent (gated DeltaNet) states.

KV pages can be shared by any request whose prompt starts with their tokens,
but a linear-attention layer's state after a prefix cannot be rebuilt from
pages: it is saved whole at one position and restored whole.  For each
prompt the scheduler ends a prefill chunk at the last page boundary before
the prompt's final token; the engine copies the sequence's state (every
linear layer's S matrix and conv window) into an entry keyed by the page-chain
hash of the prefix there.  A later request looks up the deepest boundary of
its prompt with a saved state and is admitted with a hit of exactly that many
tokens (or none, if the KV pages were evicted meanwhile); before its first
step the entry is copied into its state slot, and its prefill resumes at the
boundary.  Entries are evicted LRU.

Reference behaviour: recurrent state saved 16 tokens before the prompt's end
and restored whole (src/inference/split/prefix_cache.rs:187).
"""
from __future__ import annotations

from collections import OrderedDict

import torch


class StateCache:
    def __init__(self, kv, entries: int):
        self.kv = kv
        self.n = entries
        self.ssm = torch.zeros((kv.ssm.shape[0], entries) + tuple(kv.ssm.shape[2:]),
                               dtype=kv.ssm.dtype, device=kv.ssm.device)
        self.conv = torch.zeros((kv.conv.shape[0], entries) + tuple(kv.conv.shape[2:]),
                                dtype=kv.conv.dtype, device=kv.conv.device)
        self.of: OrderedDict[int, int] = OrderedDict()   # chain hash -> entry, LRU order
        self.saves = self.restores = 0

    def has(self, key: int) -> bool:
        return key in self.of

    def deepest(self, hashes) -> int:
        """Index of the deepest page boundary with a saved state (-1: none)."""
        for i in range(len(hashes) - 1, -1, -1):
            if int(hashes[i]) in self.of:
                return i
        return -1

    def save(self, key: int, slot: int):
        e = self.of.pop(key, None)
        if e is None:
            e = len(self.of) if len(self.of) < self.n else self.of.popitem(last=False)[1]
        self.of[key] = e
        self.ssm[:, e].copy_(self.kv.ssm[:, slot])
        self.conv[:, e].copy_(self.kv.conv[:, slot])
        self.saves += 1

    def restore(self, key: int, slot: int) -> bool:
        e = self.of.get(key)
        if e is None:
            return False
        self.of.move_to_end(key)
        self.kv.ssm[:, slot].copy_(self.ssm[:, e])
        self.kv.conv[:, slot].copy_(self.conv[:, e])
        self.restores += 1
        return True
