"""Speculative decoding with a model's own next-token-prediction (MTP) block.

Files of some families (Qwen 3.5, GLM-4.5) carry one extra decoder block after
the trunk that was trained to predict the token after next from the trunk's
final hidden state and the next token.  `MtpSpeculator` drafts a chain with it
and lets the trunk verify the chain in one forward (greedy: the output is
exactly what plain greedy decoding produces):

1. The trunk's forward gives the next token y and, for every row, its
   output-normed hidden state h.
2. The head pairs y with h at the last position and predicts d1; each further
   draft step pairs its own last draft with the head's own normed output (the
   chain of llama.cpp's speculative MTP draft), up to `depth` tokens.
3. One trunk forward over [y, d1 .. dk] gives the trunk's own choice after
   each; the longest agreeing prefix is kept plus the trunk's next token.
4. The head's cache takes in only accepted positions, paired with the trunk's
   hidden states from the verify pass -- so no rejected row stays in it -- and
   its output there starts the next draft.

Hybrid trunks (gated DeltaNet layers) carry recurrent state that a rejected
draft must not advance: the state is saved before the verify pass and, when a
draft is cut short, restored and advanced over the accepted rows again.

The head's cache holds one layer; positions are slots (one sequence, pages in
order).  CPU model only (LlamaCPU with mtp=True).  Reference: split/mtp.rs
(the head, its cache of accepted positions) and the speculative loop in
src/inference/model_worker.rs.
"""
from __future__ import annotations

import torch

from ..ops.attention import PagedKVCache
from .chain_spec import ChainSpec, SpecStats

MtpStats = SpecStats


class MtpSpeculator(ChainSpec):
    def __init__(self, model, depth: int = 3, max_len: int = 2048, page_size: int = 16):
        if model.mtp is None:
            raise ValueError("the model was loaded without its next-token-prediction block")
        super().__init__(model, max_len, page_size)
        self.depth = depth
        cfg = model.cfg
        self.kv_mtp = PagedKVCache(1, self.pages, cfg.n_kv_heads, cfg.head_dim, "cpu", page_size,
                                   dtype=torch.float32)

    def _head(self, tokens, hidden, p0):
        return self.m.mtp_forward(torch.as_tensor(tokens, dtype=torch.int32), hidden,
                                  self._batch(tokens, p0), self.kv_mtp)

    def _draft(self, first_logits, first_out, p_next: int) -> list[int]:
        """d1 (the token at position p_next) from the head's last row, then
        chained steps: d_k at position p_next + k - 1 paired with the head's
        own output there predicts d_{k+1}."""
        d = [int(first_logits[-1].argmax())]
        out = first_out[-1:]
        for k in range(1, self.depth):
            p = p_next + k - 1
            if p + 1 >= self.max_len:
                break
            lg, out = self._head([d[-1]], out, p)
            d.append(int(lg[-1].argmax()))
        return d

    def generate(self, prompt: list[int], max_new: int) -> list[int]:
        """Greedy continuation of `prompt` (max_new tokens)."""
        n = len(prompt)
        if n + max_new + self.depth + 1 > self.max_len:
            raise ValueError("prompt + tokens exceed max_len")
        logits, hidden = self._trunk(prompt, 0)
        y = int(logits[-1].argmax())
        out = [y]
        # the head over the prompt: position p pairs x_p with h_{p-1}; the last
        # row pairs the new token y with the last prompt state
        lg, hout = self._head(list(prompt[1:]) + [y], hidden, 1)
        draft = self._draft(lg, hout, n + 1)
        pos = n                          # position of y, the last committed token
        while len(out) < max_new:
            a, bonus, vhid = self._check(y, draft[: max_new - len(out)], pos)
            new = draft[:a] + [bonus]
            out += new
            # the head's cache: the committed positions pos+1 .. pos+a+1, each
            # paired with the trunk's state one position earlier
            lg, hout = self._head(new, vhid, pos + 1)
            pos += a + 1
            y = bonus
            if len(out) < max_new:
                draft = self._draft(lg, hout, pos + 1)
        return out[:max_new]
