"""Model runners: turn a scheduler StepPlan into one forward + token selection.

``GpuRunner`` (one GPU):
  * host side builds the per-row arrays (tokens, positions, KV slots,
    block-table rows, visible lengths, sampled rows) into pinned buffers and
    copies them to static device buffers with one async H2D each;
  * decode-only steps whose batch fits a captured size replay a CUDA graph of
    the whole forward (the reference's central finding is that decode is bound
    by launch count: 1,085 submissions per token, docs/invariants/inference.md:1727;
    its graphs cover 2-layer groups, src/inference/cuda_graph.rs:274 -- here the
    graph covers the entire step);
  * token selection runs on the device; only the sampled ids come back (D2H).

``CpuRunner`` runs the fp32 CPU model with the same interface.
"""
from __future__ import annotations

import numpy as np
import torch

from ..models.llama import StepBatch
from ..ops.attention import PagedKVCache
from .sampling import DeviceSampler, SamplingParams, sample_host


def plan_arrays(plan, block_manager, max_pages: int):
    """numpy per-row arrays of a StepPlan."""
    tokens = plan.tokens
    positions = plan.positions
    slots = plan.slots
    row_seq = plan.row_seq
    seq_ids = [int(s) for s in plan.seq_ids]
    bt_seq = block_manager.block_table(seq_ids, max_pages) if seq_ids else np.zeros((0, max_pages), np.int32)
    bt_rows = bt_seq[row_seq] if len(row_seq) else np.zeros((0, max_pages), np.int32)
    seq_lens = (positions + 1).astype(np.int32)
    start, ntok, samp = plan.seq_start, plan.seq_ntok, plan.seq_sample
    sample_rows = np.array([start[b] + ntok[b] - 1 for b in range(len(seq_ids)) if samp[b]],
                           dtype=np.int64)
    return tokens, positions, slots, bt_rows, seq_lens, sample_rows


class StateSlots:
    """Recurrent-state slots of the linear-attention layers, one per live
    sequence; the last slot takes graph padding rows."""

    def __init__(self, n: int):
        self.free = list(range(n - 1, -1, -1))
        self.of: dict[int, int] = {}
        self.trash = n

    def get(self, sid: int) -> int:
        s = self.of.get(sid)
        if s is None:
            if not self.free:
                raise RuntimeError("no free linear-attention state slot")
            s = self.of[sid] = self.free.pop()
        return s

    def release(self, sid: int):
        s = self.of.pop(sid, None)
        if s is not None:
            self.free.append(s)


def ssm_table(plan, positions, slots: StateSlots) -> np.ndarray:
    """int32 [S, 4] (row0, nrows, state slot, position of row0) per sequence."""
    out = np.zeros((len(plan.seq_ids), 4), np.int32)
    for b, sid in enumerate(plan.seq_ids):
        r0, n = int(plan.seq_start[b]), int(plan.seq_ntok[b])
        out[b] = (r0, n, slots.get(int(sid)), int(positions[r0]) if n else 0)
    return out


def image_rows(plan, positions, images: dict):
    """(rows int32 [n], embeddings [n, hidden]) of this step's rows that fall
    on an image's span of a prompt (images: request id -> [(first position,
    rows tensor)]), or None."""
    if not images:
        return None
    rs, pos = np.asarray(plan.row_seq), np.asarray(positions)
    idx, vals = [], []
    for si, rid in enumerate(np.asarray(plan.seq_ids)):
        spans = images.get(int(rid))
        if not spans:
            continue
        rows = np.nonzero(rs == si)[0]
        if len(rows) == 0:
            continue
        p = pos[rows]
        for p0, data in spans:
            m = (p >= p0) & (p < p0 + data.shape[0])
            if m.any():
                idx.append(rows[m])
                vals.append(data[torch.as_tensor(p[m] - p0, dtype=torch.int64, device=data.device)])
    if not idx:
        return None
    return np.concatenate(idx).astype(np.int32), torch.cat(vals)


def lora_rows(plan, lora_of: dict) -> np.ndarray:
    """int32 [N] adapter index of each token row (-1: none)."""
    per_seq = np.array([lora_of.get(int(s), -1) for s in plan.seq_ids], np.int32)
    rs = np.asarray(plan.row_seq)
    return per_seq[rs] if len(rs) else np.zeros(0, np.int32)


def attention_groups(plan, n_rep: int, seq_start=None, seq_ntok=None):
    """Row groups for the tensor-core attention kernel: runs of at most
    128 // n_rep consecutive positions of one sequence (None if every
    sequence contributes a single row, i.e. pure decode)."""
    ntok = plan.seq_ntok if plan is not None else seq_ntok
    starts = plan.seq_start if plan is not None else seq_start
    if len(ntok) == 0 or int(np.max(ntok)) <= 1:
        return None
    ppg = max(1, 128 // n_rep)
    r0, npos = [], []
    for st, n in zip(starts, ntok):
        for o in range(0, int(n), ppg):
            r0.append(int(st) + o)
            npos.append(min(ppg, int(n) - o))
    return np.asarray(r0, np.int32), np.asarray(npos, np.int32), ppg


class GpuRunner:
    def __init__(self, model, kv: PagedKVCache, max_tokens: int, max_seqs: int, max_model_len: int,
                 graph_sizes=(1, 2, 4, 8, 16, 32, 64), use_graphs: bool = True, trash_page: int = -1):
        self.model, self.kv = model, kv
        self.device = model.device
        self.max_tokens, self.max_seqs = max_tokens, max_seqs
        self.max_model_len = max_model_len
        self.max_pages = (max_model_len + kv.page_size - 1) // kv.page_size
        self.ctx = model.make_context(max_tokens, max(max_seqs, max(graph_sizes)), max_model_len)
        self.sampler = DeviceSampler(self.device, max(max_seqs, max(graph_sizes)))
        dev = self.device
        mt = max_tokens
        # static device inputs (graph-safe addresses)
        self.d_tokens = torch.zeros(mt, dtype=torch.int32, device=dev)
        self.d_pos = torch.zeros(mt, dtype=torch.int32, device=dev)
        self.d_slots = torch.zeros(mt, dtype=torch.int32, device=dev)
        self.d_bt = torch.zeros(mt, self.max_pages, dtype=torch.int32, device=dev)
        self.d_lens = torch.ones(mt, dtype=torch.int32, device=dev)
        self.d_samp = torch.zeros(mt, dtype=torch.int64, device=dev)
        # pinned host staging
        self.h_i32 = torch.zeros(4 * mt, dtype=torch.int32).pin_memory()
        self.h_bt = torch.zeros(mt, self.max_pages, dtype=torch.int32).pin_memory()
        self.h_samp = torch.zeros(mt, dtype=torch.int64).pin_memory()
        self.h_out = torch.zeros(mt, dtype=torch.int32).pin_memory()
        self.trash_page = trash_page if trash_page >= 0 else kv.num_pages - 1
        self.graph_sizes = sorted(s for s in graph_sizes if s <= min(max_tokens, max_seqs))
        self.use_graphs = use_graphs
        self.graphs: dict[int, tuple] = {}
        self.lora_of = None
        self.images: dict = {}
        self.d_lora = torch.full((mt,), -1, dtype=torch.int32, device=dev)
        self.h_lora = torch.full((mt,), -1, dtype=torch.int32).pin_memory()
        self.slots = None
        if getattr(model, "n_lin_layers", 0):
            ms = max(max_seqs, max(graph_sizes))
            self.slots = StateSlots(max_seqs)
            self.d_ssm = torch.zeros(ms, 4, dtype=torch.int32, device=dev)
            self.h_ssm = torch.zeros(ms, 4, dtype=torch.int32).pin_memory()
        self.h2d_bytes = 0
        self.d2h_bytes = 0
        self.launches_per_step = None

    # ------------------------------------------------------------------ inputs
    def _upload(self, tokens, positions, slots, bt_rows, seq_lens, sample_rows, pad_to: int = 0):
        N = len(tokens)
        M = max(N, pad_to)
        h = self.h_i32
        mt0 = self.max_tokens
        h[0:N] = torch.from_numpy(np.asarray(tokens, np.int32))
        h[mt0: mt0 + N] = torch.from_numpy(np.asarray(positions, np.int32))
        h[2 * mt0: 2 * mt0 + N] = torch.from_numpy(np.asarray(slots, np.int32))
        h[3 * mt0: 3 * mt0 + N] = torch.from_numpy(np.asarray(seq_lens, np.int32))
        self.h_bt[:N] = torch.from_numpy(bt_rows)
        S = len(sample_rows)
        self.h_samp[:S] = torch.from_numpy(sample_rows)
        if M > N:  # padding rows write to the trash page and read one key from it
            h[N:M] = 0
            h[mt0 + N: mt0 + M] = 0
            h[2 * mt0 + N: 2 * mt0 + M] = self.trash_page * self.kv.page_size
            h[3 * mt0 + N: 3 * mt0 + M] = 1
            self.h_bt[N:M] = self.trash_page
            self.h_samp[S:M] = torch.arange(S, M, dtype=torch.int64) if S < M else 0
        self.d_tokens[:M].copy_(h[0:M], non_blocking=True)
        self.d_pos[:M].copy_(h[mt0:mt0 + M], non_blocking=True)
        self.d_slots[:M].copy_(h[2 * mt0:2 * mt0 + M], non_blocking=True)
        self.d_lens[:M].copy_(h[3 * mt0:3 * mt0 + M], non_blocking=True)
        self.d_bt[:M].copy_(self.h_bt[:M], non_blocking=True)
        Sm = max(S, pad_to)
        self.d_samp[:Sm].copy_(self.h_samp[:Sm], non_blocking=True)
        self.h2d_bytes = 4 * 4 * M + 4 * M * self.max_pages + 8 * Sm
        return M, Sm

    def _upload_ssm(self, table: np.ndarray, pad_to: int = 0) -> int:
        n = len(table)
        m = max(n, pad_to)
        self.h_ssm[:n] = torch.from_numpy(table)
        if m > n:  # padding sequences: no rows; row0 past every real row keeps the table sorted
            self.h_ssm[n:m, 0] = torch.arange(1 << 30, (1 << 30) + m - n, dtype=torch.int32)
            self.h_ssm[n:m, 1] = 0
            self.h_ssm[n:m, 2] = self.slots.trash
            self.h_ssm[n:m, 3] = 0
        self.d_ssm[:m].copy_(self.h_ssm[:m], non_blocking=True)
        self.h2d_bytes += 16 * m
        return m

    def _batch(self, M: int, S: int, n_seqs: int = 0) -> StepBatch:
        b = StepBatch(self.d_tokens[:M], self.d_pos[:M], self.d_slots[:M], self.d_bt[:M],
                      self.d_lens[:M], self.d_samp[:S], self.max_model_len)
        if self.slots is not None:
            b.ssm_seqs = self.d_ssm[:n_seqs]
        if self.lora_of is not None:
            b.lora_ids = self.d_lora[:M]
        return b

    def _upload_lora(self, plan, pad_to: int = 0):
        if self.lora_of is None:
            return
        ids = lora_rows(plan, self.lora_of)
        n = len(ids)
        m = max(n, pad_to)
        self.h_lora[:n] = torch.from_numpy(ids)
        self.h_lora[n:m] = -1
        self.d_lora[:m].copy_(self.h_lora[:m], non_blocking=True)
        self.h2d_bytes += 4 * m

    # ------------------------------------------------------------------ graphs
    def capture_graphs(self):
        if not self.use_graphs:
            return
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for B in self.graph_sizes:
                b = self._batch(B, B, B)
                self._init_dummy(B)
                for _ in range(2):  # warm up (sets kernel attributes, tensor maps)
                    self.model.forward(b, self.kv, self.ctx)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=s):
                    logits = self.model.forward(b, self.kv, self.ctx)
                    out = self.sampler.greedy(logits)
                self.graphs[B] = (g, logits, out)
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)

    def _init_dummy(self, B: int):
        self.d_tokens[:B] = 0
        self.d_pos[:B] = 0
        self.d_slots[:B] = self.trash_page * self.kv.page_size
        self.d_lens[:B] = 1
        self.d_bt[:B] = self.trash_page
        self.d_samp[:B] = torch.arange(B, device=self.device)
        self.d_lora[:B] = -1
        if self.slots is not None:
            self.d_ssm[:B, 0] = torch.arange(1 << 30, (1 << 30) + B, device=self.device,
                                             dtype=torch.int32)
            self.d_ssm[:B, 1] = 0
            self.d_ssm[:B, 2] = self.slots.trash
            self.d_ssm[:B, 3] = 0

    # ------------------------------------------------------------------ step
    def run(self, plan, block_manager, params: list[SamplingParams],
            history: list | None = None) -> np.ndarray:
        """`history`: per sampled row, the request's generated-token counts
        (for frequency / presence penalties) or None."""
        tokens, positions, slots, bt_rows, seq_lens, sample_rows = plan_arrays(
            plan, block_manager, self.max_pages)
        N, S = len(tokens), len(sample_rows)
        if N == 0:
            return np.zeros(0, np.int32)
        decode_only = plan.n_prefill_tokens == 0 and N == S
        # the captured graphs end in argmax: penalized rows take the eager path
        greedy = all(p.greedy and not p.penalized for p in params)
        B = next((b for b in self.graph_sizes if b >= N), None) if decode_only else None
        table = ssm_table(plan, positions, self.slots) if self.slots is not None else None
        if B is not None and B in self.graphs and greedy:
            self._upload(tokens, positions, slots, bt_rows, seq_lens, sample_rows, pad_to=B)
            if table is not None:
                self._upload_ssm(table, pad_to=B)
            self._upload_lora(plan, pad_to=B)
            g, logits, out = self.graphs[B]
            g.replay()
            res = out[:S]
            self.last_logits = logits[:S]
        else:
            M, _ = self._upload(tokens, positions, slots, bt_rows, seq_lens, sample_rows)
            ns = self._upload_ssm(table) if table is not None else 0
            self._upload_lora(plan)
            b = self._batch(M, S, ns)
            if table is not None and len(table):
                b.ssm_max_rows = int(table[:, 1].max())
            cfg = self.model.cfg
            grp = attention_groups(plan, cfg.n_heads // cfg.n_kv_heads)
            if grp is not None:
                b.groups = (torch.from_numpy(grp[0]).to(self.device, non_blocking=True),
                            torch.from_numpy(grp[1]).to(self.device, non_blocking=True), grp[2])
            ir = image_rows(plan, positions, self.images)
            if ir is not None:
                b.embed_rows = torch.from_numpy(ir[0]).to(self.device)
                b.embed_vals = ir[1].to(self.device)
            logits = self.model.forward(b, self.kv, self.ctx)
            self.last_logits = logits
            res = self.sampler.sample(logits, params, positions[sample_rows] if S else [], history)
        self.h_out[:S].copy_(res, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        self.d2h_bytes = 4 * S
        return self.h_out[:S].numpy().copy()


class CpuRunner:
    def __init__(self, model, kv: PagedKVCache, max_model_len: int, max_seqs: int = 64):
        self.model, self.kv = model, kv
        self.max_model_len = max_model_len
        self.max_pages = (max_model_len + kv.page_size - 1) // kv.page_size
        self.slots = StateSlots(max_seqs) if getattr(model, "n_lin_layers", 0) else None

    def forward_plan(self, plan, block_manager, h_in=None):
        tokens, positions, slots, bt_rows, seq_lens, sample_rows = plan_arrays(
            plan, block_manager, self.max_pages)
        b = StepBatch(torch.from_numpy(np.asarray(tokens, np.int32)),
                      torch.from_numpy(np.asarray(positions, np.int32)),
                      torch.from_numpy(np.asarray(slots, np.int32)), torch.from_numpy(bt_rows),
                      torch.from_numpy(seq_lens), torch.from_numpy(sample_rows), self.max_model_len)
        if self.slots is not None:
            b.ssm_seqs = torch.from_numpy(ssm_table(plan, positions, self.slots))
        if getattr(self, "lora_of", None) is not None:
            b.lora_ids = torch.from_numpy(lora_rows(plan, self.lora_of))
        ir = image_rows(plan, positions, getattr(self, "images", None))
        if ir is not None:
            b.embed_rows = torch.from_numpy(ir[0])
            b.embed_vals = ir[1].cpu()
        return self.model.forward(b, self.kv, None, h_in), positions, sample_rows

    def run(self, plan, block_manager, params: list[SamplingParams],
            history: list | None = None) -> np.ndarray:
        if len(plan) == 0:
            return np.zeros(0, np.int32)
        logits, positions, sample_rows = self.forward_plan(plan, block_manager)
        self.last_logits = logits
        return sample_host(logits, params, positions[sample_rows], history)
