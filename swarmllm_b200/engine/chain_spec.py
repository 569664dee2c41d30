"""The check shared by the CPU speculators (engine/mtp.py, engine/block_spec.py):
one sequence, a chain of guessed tokens verified by one trunk forward over
[last token, guesses...]; the longest prefix the trunk agrees with is kept
plus the trunk's own next token, so greedy output equals plain decoding.

A hybrid trunk (gated DeltaNet layers) advances recurrent state over every
verified row: the state is saved before the check and, when the chain is cut
short, restored and advanced over the kept rows again.  Positions are slots
(pages in order) of the speculator's own caches.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from ..models.llama import StepBatch
from ..ops.attention import PagedKVCache


@dataclass
class SpecStats:
    rounds: int = 0
    drafted: int = 0
    accepted: int = 0

    @property
    def acceptance(self) -> float:
        return self.accepted / self.drafted if self.drafted else 0.0

    @property
    def tokens_per_round(self) -> float:
        return (self.accepted + self.rounds) / self.rounds if self.rounds else 0.0


class ChainSpec:
    def __init__(self, model, max_len: int = 2048, page_size: int = 16):
        self.m = model
        cfg = model.cfg
        self.ps = page_size
        self.max_len = max_len
        self.pages = (max_len + page_size - 1) // page_size + 1
        self.kv = PagedKVCache(model.n_kv_layers, self.pages, cfg.n_kv_heads, cfg.head_dim, "cpu",
                               page_size, dtype=torch.float32)
        spec = model.linear_state_spec()
        if spec:
            self.kv.add_linear_state(spec[0], 1, *spec[1:])
        self.bt = torch.arange(self.pages, dtype=torch.int32)
        self.stats = SpecStats()

    def _batch(self, tokens, p0: int) -> StepBatch:
        n = len(tokens)
        pos = torch.arange(p0, p0 + n, dtype=torch.int32)
        ssm = torch.tensor([[0, n, 0, p0]], dtype=torch.int32) if self.m.n_lin_layers else None
        return StepBatch(torch.as_tensor(tokens, dtype=torch.int32), pos, pos,
                         self.bt.repeat(n, 1), pos + 1, torch.arange(n), p0 + n, ssm_seqs=ssm)

    def _trunk(self, tokens, p0, capture=()):
        """Logits of every row and the output-normed hidden states."""
        return self.m.forward(self._batch(tokens, p0), self.kv, want_hidden=True, capture=capture)

    def _save_state(self):
        if self.kv.ssm is None:
            return None
        return self.kv.ssm.clone(), self.kv.conv.clone()

    def _restore_state(self, st):
        if st is not None:
            self.kv.ssm.copy_(st[0])
            self.kv.conv.copy_(st[1])

    def _check(self, y: int, guesses: list[int], pos: int, capture=()):
        """Verify `guesses` after token y at position pos: (kept guesses a,
        bonus token, trunk hidden states of rows 0..a); the trunk's caches
        and recurrent state end as after exactly y and the kept guesses."""
        st = self._save_state()
        vlog, vhid = self._trunk([y] + guesses, pos, capture)
        a = 0
        while a < len(guesses) and int(vlog[a].argmax()) == guesses[a]:
            a += 1
        bonus = int(vlog[a].argmax())
        self.stats.rounds += 1
        self.stats.drafted += len(guesses)
        self.stats.accepted += a
        if a < len(guesses) and st is not None:
            self._restore_state(st)
            self._trunk([y] + guesses[:a], pos, capture)
        return a, bonus, vhid[: a + 1]
