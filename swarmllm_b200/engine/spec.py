"""Tree speculative decoding (greedy): a small drafter grows a token tree, the
target model verifies every node in one forward, the longest path the target
agrees with is kept.

One round for a batch of sequences:
  1. drafter: rows = its pending tokens (committed last round but not yet in
     the drafter's KV) ending with the root (the last committed token); its
     top-`width` tokens at the root (tree_rank kernel: log-sum-exp + top-k on
     the device) start the tree
  2. drafter, levels 1..depth-1: one row per frontier node, visibility = the
     node's ancestors (tree attention mask), top-`width` children per node,
     the `width` best by cumulative log-probability survive (DraftTree.expand)
  3. target: one row per tree node (1 + depth*width rows per sequence), each
     seeing the context plus its ancestors; greedy token per node
  4. walk: from the root, follow the child carrying the target's token; the
     path plus the target's token at its end (the bonus) are committed
  5. both KV caches move the accepted nodes' rows to consecutive positions
     (PagedKVCache.copy_slots) and drop the rest (BlockManager.truncate)

Node i of a tree sits at logical KV index root + i (nodes are appended level
by level in index order), so the DraftTree ancestor bitmask is directly the
attention mask relative to tree_start = root.

Greedy output equals the target's own greedy decoding: every committed token
is the target's argmax given exactly the committed prefix.  With a drafter
that agrees with the target, each round commits depth + 1 tokens for one
target forward.

Sampled requests (temperature > 0) use coupled noise: the token for position
p + 1 is argmax(logits / T + g(seed, p, token)) over the top-k / top-p set,
with the Gumbel noise g drawn from Philox4x32-10 keyed by (seed, position,
token) -- the same rule the non-speculative sampler applies.  The target's
token at every tree node is its coupled sample at that node's position, so a
committed token is exactly what plain sampling would have drawn after the
same prefix: acceptance changes the speed, never the output distribution.
The drafter proposes its own coupled sample at each frontier node (with the
same seed and positions) as the first child, then its top-k tokens, so a
drafter whose distribution is close to the target's is accepted often.

Reference: the tree path of the reference's speculative executor (draft trees
with a visibility bitmask, src/inference/draft_tree.rs:92,617; verify walk,
src/inference/sampling.rs:496; KV rollback on rejection).
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field

import numpy as np
import torch

from ..models.llama import StepBatch
from ..ops.attention import PagedKVCache
from ..utils.ext import C, native
from .sampling import DeviceSampler, SamplingParams



@dataclass
class SpecStats:
    rounds: int = 0
    committed: int = 0
    accepted: int = 0       # drafted tokens the target agreed with
    seconds: float = 0.0

    @property
    def tokens_per_round(self) -> float:
        return self.committed / max(1, self.rounds)


@dataclass
class _Seq:
    sid: int
    max_new: int
    out: list = field(default_factory=list)
    pos: int = 0            # tokens in the target KV
    root: int = 0           # last committed token (in neither KV yet)
    dpos: int = 0           # tokens in the drafter KV
    pending: list = field(default_factory=list)  # committed, not yet in the drafter KV
    params: SamplingParams = field(default_factory=SamplingParams)
    stopped: bool = False   # end of sequence committed

    @property
    def done(self) -> bool:
        return self.stopped or len(self.out) >= self.max_new

    def commit(self, new: list) -> int:
        """Append committed tokens (up to max_new, through an end-of-sequence
        token); returns how many were kept."""
        room = self.max_new - len(self.out)
        new = new[:room]
        eos = self.params.eos_token_id
        if eos >= 0 and not self.params.ignore_eos and eos in new:
            new = new[:new.index(eos) + 1]
            self.stopped = True
        self.out.extend(new)
        return len(new)


class _Side:
    """One model with its paged KV cache, block manager and forward context."""

    def __init__(self, model, max_rows: int, max_samples: int, max_len: int, max_seqs: int,
                 page: int = 16):
        cfg = model.cfg
        self.model = model
        self.page = page
        self.pages_per_seq = (max_len + page - 1) // page
        pages = max_seqs * self.pages_per_seq + 1
        self.kv = PagedKVCache(model.n_kv_layers, pages, model.n_kv, cfg.head_dim,
                               model.device, page)
        self.bm = native().BlockManager(pages, page, False)
        self.ctx = model.make_context(max_rows, max_samples, max_len)
        self.max_len = max_len
        self.dev = model.device

    def phys(self, sid: int, logical) -> list[int]:
        bt = self.bm.block_table([sid], self.pages_per_seq)[0]
        return [int(bt[i // self.page]) * self.page + i % self.page for i in logical]

    def forward(self, rows: list[tuple], sample_rows: list[int], tree: bool) -> torch.Tensor:
        """rows: (sid, token, position, slot, seq_len, tree_start, mask)."""
        d = self.dev
        sids = sorted({r[0] for r in rows})
        bt_seq = dict(zip(sids, self.bm.block_table(sids, self.pages_per_seq)))
        t = lambda a, dt=torch.int32: torch.as_tensor(np.asarray(a), dtype=dt).to(d)
        b = StepBatch(t([r[1] for r in rows]), t([r[2] for r in rows]), t([r[3] for r in rows]),
                      t(np.stack([bt_seq[r[0]] for r in rows])), t([r[4] for r in rows]),
                      t(sample_rows, torch.int64), self.max_len)
        if tree:
            b.tree_start = t([r[5] for r in rows])
            b.tree_mask = t(np.asarray([r[6] for r in rows], dtype=np.uint64).view(np.int64),
                            torch.int64)
        return self.model.forward(b, self.kv, self.ctx)

    def commit_path(self, sid: int, root: int, path: list[int], keep: int):
        """Move nodes path[1:keep] (at logical root + node) to root + 1.. and
        truncate the sequence after them."""
        if keep > 1:
            src = self.phys(sid, [root + n for n in path[1:keep]])
            dst = self.phys(sid, [root + i for i in range(1, keep)])
            if src != dst:
                self.kv.copy_slots(torch.tensor(src, device=self.dev),
                                   torch.tensor(dst, device=self.dev))
        self.bm.truncate(sid, root + keep)


def walk_constrained(tree, target: list, logits, params: SamplingParams):
    """The verify walk of a constrained reply (JSON / schema): at each node on
    the path the committed token is what plain constrained decoding commits
    there -- the target's token if the constraint allows it, else the best
    allowed candidate of that node's logits -- and the walk follows the child
    carrying it.  Every committed token (path nodes and the bonus) is told to
    the constraint once, in order, so the reply equals plain constrained
    decoding.  Reference: src/inference/reply_grammar.rs:334
    (guesses_it_allows: a check carries only the guesses the grammar allows)."""
    from .sampling import constrained_token
    parents, toks = tree.parents(), tree.tokens()
    child = {}
    for i in range(1, len(toks)):
        child.setdefault((parents[i], toks[i]), i)   # first match, as DraftTree.walk
    path, cur = [0], 0
    while True:
        t = constrained_token(params.constraint, int(target[cur]), logits[cur],
                              params.eos_token_id)
        nxt = child.get((cur, t))
        if nxt is None:
            return path, t
        path.append(nxt)
        cur = nxt


class TreeSpecDecoder:
    # constrained replies are verified by walk_constrained
    constrained = True

    def __init__(self, target, drafter, depth: int = 4, width: int = 4, max_seqs: int = 32,
                 max_model_len: int = 4096, prefill_chunk: int = 2048):
        assert 1 + depth * width <= 64, "tree masks are 64-bit: at most 64 nodes"
        assert target.cfg.vocab == drafter.cfg.vocab, "drafter and target share a vocabulary"
        self.depth, self.width = depth, width
        self.n_nodes = 1 + depth * width
        self.chunk = prefill_chunk
        ml = max_model_len + self.n_nodes + 16
        self.t = _Side(target, max(prefill_chunk, max_seqs * self.n_nodes),
                       max_seqs * self.n_nodes, ml, max_seqs)
        self.d = _Side(drafter, max(prefill_chunk, max_seqs * (width + 2)), max_seqs * width,
                       ml, max_seqs)
        self.stats = SpecStats()
        self._next_sid = 0
        rows = max_seqs * width
        V = drafter.cfg.vocab
        dev = drafter.device
        self._rk_ids = torch.zeros(rows * width, dtype=torch.int32, device=dev)
        self._rk_lp = torch.zeros(rows * width, dtype=torch.float32, device=dev)
        self._rk_ws = torch.zeros(int(C().tree_rank_ws_floats(rows, V, width)),
                                  dtype=torch.float32, device=dev)
        self.t_sampler = DeviceSampler(target.device, max_seqs * self.n_nodes)
        self.d_sampler = DeviceSampler(dev, rows + max_seqs)

    def _rank(self, logits: torch.Tensor):
        """Top-`width` (log-prob, token) per row on the device (tree_rank kernel)."""
        n, W = logits.shape[0], self.width
        C().tree_rank(logits, W, self._rk_ids, self._rk_lp, self._rk_ws)
        return (self._rk_lp[:n * W].view(n, W).cpu().numpy(),
                self._rk_ids[:n * W].view(n, W).cpu().numpy())

    # ------------------------------------------------------------------ prefill
    def _prefill(self, side: _Side, sid: int, prompt: list[int]) -> torch.Tensor:
        side.bm.add_sequence(sid, prompt)
        slots = list(side.bm.append_slots(sid, len(prompt)))
        logits = None
        for c0 in range(0, len(prompt), self.chunk):
            c1 = min(len(prompt), c0 + self.chunk)
            rows = [(sid, prompt[i], i, slots[i], i + 1, 0, 0) for i in range(c0, c1)]
            logits = side.forward(rows, [c1 - c0 - 1], tree=False)
        return logits

    def add(self, prompt: list[int], max_new: int, params: SamplingParams | None = None) -> _Seq:
        sid = self._next_sid
        self._next_sid += 1
        s = _Seq(sid, max_new, params=params or SamplingParams())
        lg = self._prefill(self.t, sid, prompt)
        self._prefill(self.d, sid, prompt)
        s.root = int(self.t_sampler.sample(lg[:1], [s.params], [len(prompt) - 1])[0])
        if s.params.constraint is not None:
            from .sampling import constrained_token
            s.root = constrained_token(s.params.constraint, s.root, lg[0], s.params.eos_token_id)
        s.commit([s.root])
        s.pos = s.dpos = len(prompt)
        return s

    def _proposals(self, logits, seqs_rows: list, positions: list):
        """Candidate children per drafter row: its top-`width` tokens by
        log-probability, with the row's coupled sample first for sampled
        requests (given log-probability 0 so the tree keeps that branch)."""
        v, ix = self._rank(logits)
        params = [s.params for s in seqs_rows]
        if all(p.greedy for p in params):
            return v, ix
        samp = self.d_sampler.sample(logits, params, positions).cpu().numpy()
        W = self.width
        for r, p in enumerate(params):
            if p.greedy:
                continue
            tok = int(samp[r])
            rest = [(float(lp), int(t)) for lp, t in zip(v[r], ix[r]) if int(t) != tok][:W - 1]
            ix[r] = [tok] + [t for _, t in rest]
            v[r] = [0.0] + [lp for lp, _ in rest]
        return v, ix

    # ------------------------------------------------------------------ one round
    def _draft(self, seqs: list[_Seq]):
        W, D = self.width, self.depth
        rows, samp, roots = [], [], {}
        for s in seqs:
            toks = s.pending + [s.root]
            slots = list(self.d.bm.append_slots(s.sid, len(toks)))
            for j, tok in enumerate(toks):
                p = s.dpos + j
                rows.append((s.sid, tok, p, slots[j], p + 1, 0, 0))
            samp.append(len(rows) - 1)
            roots[s.sid] = s.dpos + len(toks) - 1
        v, ix = self._proposals(self.d.forward(rows, samp, tree=False), seqs,
                                [roots[s.sid] for s in seqs])
        trees, fronts = {}, {}
        for n, s in enumerate(seqs):
            tr = native().DraftTree(s.root, self.n_nodes)
            fronts[s.sid] = tr.expand(ix[n].tolist(), v[n].tolist(), W, W)
            trees[s.sid] = tr
        for _ in range(1, D):
            rows, owners = [], []
            for s in seqs:
                tr, fr, r = trees[s.sid], fronts[s.sid], roots[s.sid]
                slots = list(self.d.bm.append_slots(s.sid, len(fr)))
                masks, toks, deps = tr.masks(), tr.tokens(), tr.depths()
                for j, node in enumerate(fr):
                    rows.append((s.sid, toks[node], r + deps[node], slots[j], r + len(tr), r,
                                 int(masks[node])))
                    owners.append(s)
            v, ix = self._proposals(self.d.forward(rows, list(range(len(rows))), tree=True),
                                    owners, [row[2] for row in rows])
            k0 = 0
            for s in seqs:
                tr, nf = trees[s.sid], len(fronts[s.sid])
                fronts[s.sid] = tr.expand(ix[k0:k0 + nf].reshape(-1).tolist(),
                                          v[k0:k0 + nf].reshape(-1).tolist(), W, W)
                k0 += nf
        return trees, roots

    def step(self, seqs: list[_Seq]):
        seqs = [s for s in seqs if not s.done]
        if not seqs:
            return
        t0 = time.perf_counter()
        trees, droots = self._draft(seqs)
        self.last_draft_s = time.perf_counter() - t0
        # ---- verify every node with the target
        rows, rparams = [], []
        for s in seqs:
            tr = trees[s.sid]
            n = len(tr)
            slots = list(self.t.bm.append_slots(s.sid, n))
            masks, toks, deps = tr.masks(), tr.tokens(), tr.depths()
            for i in range(n):
                rows.append((s.sid, toks[i], s.pos + deps[i], slots[i], s.pos + n, s.pos,
                             int(masks[i])))
                rparams.append(s.params)
        logits = self.t.forward(rows, list(range(len(rows))), tree=True)
        # the target's token at every node: argmax, or its coupled sample at that position
        tgt = self.t_sampler.sample(logits, rparams, [r[2] for r in rows]).cpu().numpy()
        k0 = 0
        for s in seqs:
            tr = trees[s.sid]
            n = len(tr)
            if s.params.constraint is not None:
                path, bonus = walk_constrained(tr, tgt[k0:k0 + n].tolist(), logits[k0:k0 + n],
                                               s.params)
            else:
                path, bonus = tr.walk(tgt[k0:k0 + n].tolist())
            k0 += n
            toks = tr.tokens()
            new = [toks[i] for i in path[1:]] + [bonus]
            # target: root + accepted nodes now sit at pos .. pos + len(path) - 1
            self.t.commit_path(s.sid, s.pos, path, len(path))
            # drafter: nodes of depth < depth have drafter KV (the last level was never fed)
            r = droots[s.sid]
            keep = min(len(path), self.depth)
            self.d.commit_path(s.sid, r, path, keep)
            s.dpos = r + keep
            s.pending = [toks[i] for i in path[keep:]]
            s.pos += len(path)
            s.root = bonus
            self.stats.committed += s.commit(new)
            self.stats.accepted += len(path) - 1
        self.stats.rounds += 1
        self.stats.seconds += time.perf_counter() - t0

    def free(self, s: _Seq):
        self.t.bm.free_sequence(s.sid)
        self.d.bm.free_sequence(s.sid)

    def generate(self, prompts: list[list[int]], max_new: int,
                 params: SamplingParams | None = None) -> list[list[int]]:
        seqs = [self.add(p, max_new, params) for p in prompts]
        while any(not s.done for s in seqs):
            self.step(seqs)
        for s in seqs:
            self.free(s)
        return [s.out for s in seqs]
