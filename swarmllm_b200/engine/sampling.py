"""Sampling parameters and token selection.

Greedy and temperature/top-k/top-p sampling run on the device
(``sampling.cu``); the CPU backend mirrors them with the same Philox noise
definition so a CPU run and a GPU run with the same seed pick the same
tokens up to logit rounding.  Reference: src/inference/sampling.rs:314,339.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from ..utils.ext import C


@dataclass
class SamplingParams:
    max_tokens: int = 16
    temperature: float = 0.0     # <= 0 -> greedy
    top_k: int = 0
    top_p: float = 1.0
    seed: int = 0
    eos_token_id: int = -1
    ignore_eos: bool = False
    frequency_penalty: float = 0.0   # per occurrence in the completion so far
    presence_penalty: float = 0.0    # once for any token the completion contains
    # token id -> value added to its logit before sampling (OpenAI logit_bias)
    logit_bias: dict = field(default=None, compare=False, repr=False)
    # per-request token filter applied before a token is committed (serve/json_guard.py):
    # .choose(drawn, candidates) -> token or None, .accept(token)
    constraint: object = field(default=None, compare=False, repr=False)

    @property
    def greedy(self) -> bool:
        return self.temperature <= 0.0

    @property
    def penalized(self) -> bool:
        """The logits are adjusted before sampling (penalties or logit bias)."""
        return self.frequency_penalty != 0.0 or self.presence_penalty != 0.0 or bool(self.logit_bias)


def penalty_table(params: list[SamplingParams], history: list | None):
    """CSR table (row offsets int32 [S + 1], tokens int32, values f32) of the
    logit adjustments of each sampled row, subtracted from the raw logits
    before temperature: for every distinct token t the request generated so
    far (the prompt excluded), count(t) * frequency_penalty +
    presence_penalty; minus the request's logit_bias for t.  None when no row
    is adjusted.
    Reference behaviour: src/inference/sampling.rs:75-125."""
    if not any(p.penalized for p in params):
        return None
    if history is None:
        history = [None] * len(params)
    off, tok, val = [0], [], []
    for p, h in zip(params, history):
        row: dict = {}
        if h and (p.frequency_penalty != 0.0 or p.presence_penalty != 0.0):
            for t, c in h.items():
                row[int(t)] = c * p.frequency_penalty + p.presence_penalty
        for t, b in (p.logit_bias or {}).items():     # a bias adds: subtract its negative
            row[int(t)] = row.get(int(t), 0.0) - float(b)
        tok.extend(row.keys())
        val.extend(row.values())
        off.append(len(tok))
    if not tok:      # nothing to adjust (no history yet, no bias)
        return None
    return (np.asarray(off, np.int32), np.asarray(tok, np.int32), np.asarray(val, np.float32))


class DeviceSampler:
    """Batched token selection for up to `max_rows` rows per step."""

    def __init__(self, device, max_rows: int):
        self.device = torch.device(device)
        self.out = torch.zeros(max_rows, dtype=torch.int32, device=device)
        self.temp = torch.zeros(max_rows, dtype=torch.float32, device=device)
        self.top_k = torch.zeros(max_rows, dtype=torch.int32, device=device)
        self.top_p = torch.ones(max_rows, dtype=torch.float32, device=device)
        self.seeds = torch.zeros(max_rows, dtype=torch.int64, device=device)
        self.pos = torch.zeros(max_rows, dtype=torch.int32, device=device)
        self.h_params = torch.zeros(max_rows, 5, dtype=torch.float64).pin_memory()

    def greedy(self, logits: torch.Tensor) -> torch.Tensor:
        S = logits.shape[0]
        out = self.out[:S]
        C().argmax(logits, out, None)
        return out

    def sample(self, logits: torch.Tensor, params: list[SamplingParams], positions: np.ndarray,
               history: list | None = None) -> torch.Tensor:
        S = logits.shape[0]
        pen = penalty_table(params, history)
        if pen is not None:
            d = [torch.from_numpy(a).to(self.device, non_blocking=True) for a in pen]
            C().apply_penalties(logits, *d)
        if all(p.greedy for p in params):
            return self.greedy(logits)
        t = torch.tensor([p.temperature for p in params], dtype=torch.float32)
        k = torch.tensor([p.top_k for p in params], dtype=torch.int32)
        pp = torch.tensor([p.top_p for p in params], dtype=torch.float32)
        sd = torch.tensor([p.seed for p in params], dtype=torch.int64)
        ps = torch.from_numpy(np.asarray(positions, dtype=np.int32))
        self.temp[:S].copy_(t, non_blocking=True)
        self.top_k[:S].copy_(k, non_blocking=True)
        self.top_p[:S].copy_(pp, non_blocking=True)
        self.seeds[:S].copy_(sd, non_blocking=True)
        self.pos[:S].copy_(ps, non_blocking=True)
        out = self.out[:S]
        C().sample(logits, self.temp[:S], self.top_k[:S], self.top_p[:S], self.seeds[:S],
                   self.pos[:S], out)
        return out


# --------------------------------------------------------------------------- host mirror
def philox_uniform_host(seed: int, position: int, tokens: np.ndarray) -> np.ndarray:
    """Philox4x32-10 uniforms, bit-identical to the device definition."""
    M0, M1, W0, W1 = 0xD2511F53, 0xCD9E8D57, 0x9E3779B9, 0xBB67AE85
    mask = 0xFFFFFFFF
    tok = np.asarray(tokens, dtype=np.uint64)
    c0 = tok.copy()
    c1 = np.full_like(tok, position & mask)
    c2 = np.full_like(tok, 0x5EED)
    c3 = np.zeros_like(tok)
    k0, k1 = seed & mask, (seed >> 32) & mask
    for _ in range(10):
        p0 = M0 * c0
        p1 = M1 * c2
        hi0, lo0 = (p0 >> 32) & mask, p0 & mask
        hi1, lo1 = (p1 >> 32) & mask, p1 & mask
        c0, c1, c2, c3 = (hi1 ^ c1 ^ k0) & mask, lo1, (hi0 ^ c3 ^ k1) & mask, lo0
        k0, k1 = (k0 + W0) & mask, (k1 + W1) & mask
    return (((c0 >> 8).astype(np.float64) + 0.5) / 16777216.0).astype(np.float32)


def sample_host(logits: torch.Tensor, params: list[SamplingParams], positions,
                history: list | None = None) -> np.ndarray:
    """CPU token selection with the same rules as the device kernel."""
    out = np.zeros(logits.shape[0], dtype=np.int32)
    L = logits.detach().to(torch.float32).cpu().numpy().copy()
    pen = penalty_table(params, history)
    if pen is not None:
        off, tok, val = pen
        for r in range(len(params)):
            t, v = tok[off[r]:off[r + 1]], val[off[r]:off[r + 1]]
            ok = (t >= 0) & (t < L.shape[1])
            L[r, t[ok]] -= v[ok]
    for r, p in enumerate(params):
        row = L[r]
        if p.greedy:
            out[r] = int(np.argmax(row))
            continue
        z = (row - row.max()) / p.temperature
        keep = np.ones_like(row, dtype=bool)
        if 0 < p.top_k < row.size:
            kth = np.partition(row, -p.top_k)[-p.top_k]
            keep &= row >= kth
        if p.top_p < 1.0:
            pr = np.where(keep, np.exp(z), 0.0)
            pr /= pr.sum()
            order = np.argsort(-pr)
            cum = np.cumsum(pr[order])
            cut = np.searchsorted(cum, p.top_p) + 1
            thr = pr[order[min(cut, len(order)) - 1]]
            keep &= pr >= thr
        u = philox_uniform_host(p.seed, int(positions[r]), np.arange(row.size))
        g = -np.log(-np.log(u))
        out[r] = int(np.argmax(np.where(keep, z + g, -np.inf)))
    return out


# allowed-token search of a constrained reply: the top logits first, then the row
CONSTRAINT_CANDIDATES = 64


def constrained_token(c, drawn: int, row, eos: int) -> int:
    """The token a constrained reply commits at one position: the drawn token
    if the constraint allows it, else the best allowed candidate by logit
    (the top 64, then the whole row); end of sequence when nothing keeps the
    text valid.  The constraint is told the token (c.accept)."""
    import torch
    row = row.float()
    top = torch.topk(row, min(CONSTRAINT_CANDIDATES, row.numel())).indices.tolist()
    t = c.choose(int(drawn), top)
    if t is None:
        t = c.choose(int(drawn), torch.argsort(row, descending=True).tolist())
    if t is None:
        t = eos if eos >= 0 else int(drawn)
    c.accept(t)
    return int(t)
