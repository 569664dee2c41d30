"""Paged KV cache and the attention op wrapper.

Cache layout per layer: K and V as ``[pages, n_kv, page_size, head_dim]``
fp16, 16-token pages.  A (page, kv head) is one contiguous 4 KB run
(head_dim 128), which is what the attention kernel streams.
"""
from __future__ import annotations

import torch

from ..utils.ext import C


class PagedKVCache:
    def __init__(self, n_layers: int, num_pages: int, n_kv: int, head_dim: int, device,
                 page_size: int = 16, dtype=torch.float16):
        self.n_layers, self.num_pages, self.n_kv = n_layers, num_pages, n_kv
        self.head_dim, self.page_size = head_dim, page_size
        self.data = torch.zeros(n_layers, 2, num_pages, n_kv, page_size, head_dim, dtype=dtype,
                                device=device)

    def k(self, layer: int) -> torch.Tensor:
        return self.data[layer, 0]

    def v(self, layer: int) -> torch.Tensor:
        return self.data[layer, 1]

    @staticmethod
    def bytes_per_page(n_layers: int, n_kv: int, head_dim: int, page_size: int = 16) -> int:
        return n_layers * 2 * n_kv * page_size * head_dim * 2

    def copy_slots(self, src_slots: torch.Tensor, dst_slots: torch.Tensor):
        """Move KV rows between slots in every layer (draft-tree compaction)."""
        if src_slots.numel() == 0:
            return
        ps = self.page_size
        sp, so = src_slots // ps, src_slots % ps
        dp, do = dst_slots // ps, dst_slots % ps
        d = self.data
        rows = d[:, :, sp, :, so, :].clone()  # [L, 2, n, n_kv, hd]
        d[:, :, dp, :, do, :] = rows


class AttentionWorkspace:
    """Split-KV partial buffers for the decode attention kernel."""

    def __init__(self, device, max_rows: int, n_q: int, n_kv: int, head_dim: int, max_len: int,
                 num_sms: int = 148, max_splits: int = 32):
        self.max_rows, self.max_splits, self.max_len = max_rows, max_splits, max_len
        worst = 0
        t = 1
        while True:
            tt = min(t, max_rows)
            worst = max(worst, tt * split_plan(tt, n_kv, max_len, num_sms, max_splits)[1])
            if tt == max_rows:
                break
            t *= 2
        worst *= 2  # T * n_splits(T) between powers of two is at most twice the sampled max
        self.part_o = torch.empty(worst * n_q * head_dim, dtype=torch.float32, device=device)
        self.part_ml = torch.empty(worst * n_q * 2, dtype=torch.float32, device=device)
        self.n_q, self.head_dim = n_q, head_dim


def split_plan(n_rows: int, n_kv: int, max_len: int, num_sms: int = 148,
               max_splits: int = 32) -> tuple[int, int]:
    """(keys_per_split, n_splits): enough CTAs to fill the GPU, at most
    max_splits, and a shared-memory score buffer that fits."""
    max_len = max(16, (max_len + 15) // 16 * 16)
    ctas = max(1, n_rows * n_kv)
    want = max(1, min(max_splits, (4 * num_sms + ctas - 1) // ctas))
    kps = (max_len + want - 1) // want
    kps = max(64, (kps + 15) // 16 * 16)
    kps = min(kps, 4096)
    n = (max_len + kps - 1) // kps
    if n > max_splits:
        kps = (max_len + max_splits - 1) // max_splits
        kps = (kps + 15) // 16 * 16
        n = (max_len + kps - 1) // kps
    return kps, n


def paged_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                    block_table: torch.Tensor, seq_lens: torch.Tensor, ws: AttentionWorkspace,
                    out: torch.Tensor, max_len: int, scale: float, window: int = 0,
                    sinks: torch.Tensor | None = None, softcap: float = 0.0,
                    tree_mask: torch.Tensor | None = None, tree_start: torch.Tensor | None = None,
                    num_sms: int = 148):
    """q [T, n_q, d] fp16 -> out [T, n_q, d] fp16 over paged K/V.

    Row t sees keys [0, seq_lens[t]) of its block table row (minus the
    sliding window, plus the tree mask for keys at/after tree_start[t])."""
    T, n_q, d = q.shape
    n_kv = k_cache.shape[1]
    kps, ns = split_plan(T, n_kv, max_len, num_sms, ws.max_splits)
    part_o = ws.part_o[: T * n_q * ns * d].view(T, n_q, ns, d)
    part_ml = ws.part_ml[: T * n_q * ns * 2].view(T, n_q, ns, 2)
    C().decode_attn(q, k_cache, v_cache, block_table, seq_lens, tree_mask, tree_start, sinks,
                    window, scale, softcap, kps, part_o, part_ml, out)
