"""Speculative decoding with a block drafter (DFlash, models/dflash.py) on
the CPU model: the drafter guesses block_size - 1 tokens in one forward from
the target's captured streams; the trunk verifies them as one chain
(engine/chain_spec.py), so greedy output equals plain decoding.  The drafter
takes in only committed positions (its context rows come from the trunk's
verify pass), as the reference's split/block_drafter.rs keeps them.
"""
from __future__ import annotations

import torch

from .chain_spec import ChainSpec


class BlockSpeculator(ChainSpec):
    def __init__(self, model, drafter, max_len: int = 2048, page_size: int = 16):
        super().__init__(model, max_len, page_size)
        self.d = drafter
        self.capture = tuple(drafter.cfg.target_layers)

    def generate(self, prompt: list[int], max_new: int) -> list[int]:
        """Greedy continuation of `prompt` (max_new tokens)."""
        n = len(prompt)
        if n + max_new + self.d.cfg.block_size + 1 > self.max_len:
            raise ValueError("prompt + tokens exceed max_len")
        self.d.reset()
        logits, _ = self._trunk(prompt, 0, self.capture)
        self.d.add_context(self.m.captured, slice(0, n), torch.arange(n))
        y = int(logits[-1].argmax())
        out, pos = [y], n               # y sits at position n; the drafter has 0..n-1
        while len(out) < max_new:
            guesses = self.d.draft(y, pos)[: max_new - len(out)]
            a, bonus, _ = self._check(y, guesses, pos, self.capture)
            # the committed rows y, d1..da: positions pos .. pos+a
            self.d.add_context(self.m.captured, slice(0, a + 1), torch.arange(pos, pos + a + 1))
            out += guesses[:a] + [bonus]
            pos += a + 1
            y = bonus
        return out[:max_new]
