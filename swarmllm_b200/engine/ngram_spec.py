"""N-gram (prompt lookup) speculative decoding, greedy: no drafter model.
The draft for a sequence is what followed the most recent earlier occurrence
of its longest recent n-gram (its own prompt and output are the lookup
table), so repetitive text -- code edits, quoting, extraction, structured
output -- commits several tokens per target forward.

One round for a batch of sequences:
  1. draft: for n = max_ngram .. 1, find the last earlier occurrence of the
     context's final n tokens; the (up to `depth`) tokens after it form a
     chain below the root (the last committed token)
  2. target: one row per chain node, node i seeing the context and nodes
     0..i (the tree-attention mask of a chain), greedy token per node
  3. accept the chain while the target's token at node i equals node i + 1;
     the target's token after the last accepted node is the bonus
  4. the accepted nodes already sit at consecutive KV positions: the target
     sequence is truncated after them

Output equals the target's own greedy decoding.  A sequence with no match
runs a plain decode step (a chain of one node).  Sampled requests compare the
chain with the target's coupled samples (Philox noise keyed by seed and
position, as in engine/spec.py), so their output is what plain sampling
draws.

Reference behaviour: n-gram lookup speculation (src/inference/ngram_lookup.rs:62,
model_worker.rs:4131 ngram_spec_round).
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field

import numpy as np  # noqa: F401

from .sampling import DeviceSampler, SamplingParams
from .spec import SpecStats, _Side, _Seq


def ngram_draft(ctx, max_ngram: int, depth: int, min_ngram: int = 1) -> list[int]:
    """Up to `depth` tokens that followed the most recent earlier occurrence
    of the longest suffix of `ctx` (max_ngram down to min_ngram tokens)."""
    a = np.asarray(ctx, dtype=np.int64)
    L = a.size
    for n in range(min(max_ngram, L - 1), min_ngram - 1, -1):
        # windows starting at 0 .. L - n - 1: earlier than the suffix itself
        win = np.lib.stride_tricks.sliding_window_view(a[:L - 1], n)
        hit = np.nonzero((win == a[L - n:]).all(axis=1))[0]
        if hit.size:
            st = int(hit[-1]) + n
            return a[st:st + depth].tolist()
    return []


@dataclass
class _NSeq(_Seq):
    ctx: list = field(default_factory=list)   # prompt + committed tokens (the lookup table)


class NgramSpecDecoder:
    def __init__(self, target, depth: int = 5, max_ngram: int = 3, max_seqs: int = 32,
                 max_model_len: int = 4096, prefill_chunk: int = 2048):
        assert depth + 1 <= 64, "tree masks are 64-bit"
        self.depth, self.max_ngram = depth, max_ngram
        self.chunk = prefill_chunk
        n_nodes = depth + 1
        self.t = _Side(target, max(prefill_chunk, max_seqs * n_nodes), max_seqs * n_nodes,
                       max_model_len + n_nodes + 16, max_seqs)
        self.stats = SpecStats()
        self._next_sid = 0
        self.t_sampler = DeviceSampler(target.device, max_seqs * n_nodes)

    def add(self, prompt: list[int], max_new: int, params: SamplingParams | None = None) -> _NSeq:
        sid = self._next_sid
        self._next_sid += 1
        side = self.t
        side.bm.add_sequence(sid, prompt)
        slots = list(side.bm.append_slots(sid, len(prompt)))
        lg = None
        for c0 in range(0, len(prompt), self.chunk):
            c1 = min(len(prompt), c0 + self.chunk)
            rows = [(sid, prompt[i], i, slots[i], i + 1, 0, 0) for i in range(c0, c1)]
            lg = side.forward(rows, [c1 - c0 - 1], tree=False)
        s = _NSeq(sid, max_new, pos=len(prompt), ctx=list(prompt))
        if params is not None:
            s.params = params
        s.root = int(self.t_sampler.sample(lg[:1], [s.params], [len(prompt) - 1])[0])
        s.commit([s.root])
        s.ctx.append(s.root)
        return s

    def step(self, seqs: list[_NSeq]):
        seqs = [s for s in seqs if not s.done]
        if not seqs:
            return
        t0 = time.perf_counter()
        rows, chains, rparams = [], {}, []
        for s in seqs:
            room = s.max_new - len(s.out)
            chain = [s.root] + ngram_draft(s.ctx, self.max_ngram, min(self.depth, room))
            n = len(chain)
            slots = list(self.t.bm.append_slots(s.sid, n))
            for i, tok in enumerate(chain):
                rows.append((s.sid, tok, s.pos + i, slots[i], s.pos + n, s.pos, (1 << (i + 1)) - 1))
                rparams.append(s.params)
            chains[s.sid] = chain
        logits = self.t.forward(rows, list(range(len(rows))), tree=True)
        tgt = self.t_sampler.sample(logits, rparams, [r[2] for r in rows]).cpu().numpy()
        k0 = 0
        for s in seqs:
            chain = chains[s.sid]
            n = len(chain)
            t = tgt[k0:k0 + n].tolist()
            k0 += n
            k = 0
            while k + 1 < n and chain[k + 1] == t[k]:
                k += 1
            new = chain[1:k + 1] + [t[k]]
            self.t.bm.truncate(s.sid, s.pos + k + 1)
            s.pos += k + 1
            s.root = t[k]
            kept = s.commit(new)
            s.ctx.extend(new[:kept])
            self.stats.committed += kept
            self.stats.accepted += k
        self.stats.rounds += 1
        self.stats.seconds += time.perf_counter() - t0

    def free(self, s: _NSeq):
        self.t.bm.free_sequence(s.sid)

    def generate(self, prompts: list[list[int]], max_new: int,
                 params: SamplingParams | None = None) -> list[list[int]]:
        seqs = [self.add(p, max_new, params) for p in prompts]
        while any(not s.done for s in seqs):
            self.step(seqs)
        for s in seqs:
            self.free(s)
        return [s.out for s in seqs]
