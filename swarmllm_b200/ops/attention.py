"""Paged KV cache and the attention op wrapper.

Cache layout per layer: K and V as ``[pages, n_kv, page_size, head_dim]``
fp16, 16-token pages.  A (page, kv head) is one contiguous 4 KB run
(head_dim 128), which is what the attention kernel streams.
"""
from __future__ import annotations

import functools

import torch

from ..utils.ext import C


class PagedKVCache:
    def __init__(self, n_layers: int, num_pages: int, n_kv: int, head_dim: int, device,
                 page_size: int = 16, dtype=torch.float16):
        self.n_layers, self.num_pages, self.n_kv = n_layers, num_pages, n_kv
        self.head_dim, self.page_size = head_dim, page_size
        self.data = torch.zeros(n_layers, 2, num_pages, n_kv, page_size, head_dim, dtype=dtype,
                                device=device)

        self.ssm = self.conv = None

    def add_linear_state(self, n_layers: int, slots: int, nv: int, dk: int, dv: int,
                         conv_channels: int, conv_k: int):
        """Recurrent state of the linear-attention (gated DeltaNet) layers:
        per layer and sequence slot, S [nv][dk][dv] and the conv window
        [conv_k - 1][channels], fp32."""
        dev, dt = self.data.device, torch.float32
        self.ssm = torch.zeros(n_layers, slots, nv, dk, dv, dtype=dt, device=dev)
        self.conv = torch.zeros(n_layers, slots, conv_k - 1, conv_channels, dtype=dt, device=dev)

    def ssm_state(self, layer: int) -> torch.Tensor:
        return self.ssm[layer]

    def conv_state(self, layer: int) -> torch.Tensor:
        return self.conv[layer]

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


@functools.lru_cache(maxsize=4096)
def tc_split_plan(n_groups: int, n_kv: int, max_len: int, num_sms: int = 148,
                  max_splits: int = 32) -> tuple[int, int]:
    """(keys_per_split, n_splits) for the tcgen05 kernel (one CTA per SM, whole
    128-key tiles): the split count that minimises waves x (tiles per CTA + 1),
    the +1 standing for a CTA's fixed start-up (TMEM, barriers, Q and first
    K/V loads).  Fewer splits win ties (less combine work)."""
    tiles = max(1, (max_len + 127) // 128)
    ctas = max(1, n_groups * n_kv)
    best = None
    for want in range(1, min(tiles, max_splits) + 1):
        tps = (tiles + want - 1) // want
        ns = (tiles + tps - 1) // tps
        waves = (ctas * ns + num_sms - 1) // num_sms
        cost = waves * (tps + 1)
        if best is None or cost < best[0]:
            best = (cost, tps, ns)
    return best[1] * 128, best[2]


class AttentionWorkspace:
    """Split-KV partial buffers and status word for the attention kernels."""

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
        # the tensor-core plan is not monotone in T: take its exact maximum
        worst = max(worst, max(tt * tc_split_plan(tt, n_kv, max_len, num_sms, max_splits)[1]
                               for tt in range(1, max_rows + 1)))
        self.part_o = torch.empty(worst * n_q * head_dim, dtype=torch.float32, device=device)
        self.part_ml = torch.empty(worst * n_q * 2, dtype=torch.float32, device=device)
        self.n_q, self.head_dim = n_q, head_dim
        self.status = torch.zeros(8, dtype=torch.int32, device=device)
        self.arange = torch.arange(max_rows, dtype=torch.int32, device=device)
        self.ones = torch.ones(max_rows, dtype=torch.int32, device=device)
        self.num_sms = num_sms
        self.max_splits = max_splits


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


def tc_supported(n_q: int, n_kv: int, d: int, softcap: float = 0.0) -> bool:
    return softcap == 0.0 and d in (64, 128, 256) and n_q % n_kv == 0 and n_q // n_kv <= 128


def paged_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                    block_table: torch.Tensor, seq_lens: torch.Tensor, ws: AttentionWorkspace,
                    out: torch.Tensor, max_len: int, scale: float, window: int = 0,
                    sinks: torch.Tensor | None = None, softcap: float = 0.0,
                    tree_mask: torch.Tensor | None = None, tree_start: torch.Tensor | None = None,
                    num_sms: int = 148, groups=None, force_simt: bool = False):
    """q [T, n_q, d] fp16 -> out [T, n_q, d] fp16 over paged K/V.

    Row t sees keys [0, seq_lens[t]) of its block table row (minus the
    sliding window, plus the tree mask for keys at/after tree_start[t]).
    `groups` = (row0 int32[G], npos int32[G], positions_per_group): runs of
    consecutive positions of one sequence that share a CTA on the tensor-core
    path (prefill chunks, tree rows); None = every row alone (decode)."""
    T, n_q, d = q.shape
    n_kv = k_cache.shape[1]
    if not force_simt and tc_supported(n_q, n_kv, d, softcap):
        if groups is None:
            groups = (ws.arange[:T], ws.ones[:T], 1)
        row0, npos, ppg = groups
        G = row0.shape[0]
        if ppg > 1:  # multi-position groups (prefill/tree): no key splits
            kps, ns = (max_len + 127) // 128 * 128, 1
        else:
            kps, ns = tc_split_plan(G, n_kv, max_len, num_sms, ws.max_splits)
        part_o = ws.part_o[: T * n_q * ns * d].view(T, n_q, ns, d)
        part_ml = ws.part_ml[: T * n_q * ns * 2].view(T, n_q, ns, 2)
        C().attn_tc(q, k_cache, v_cache, row0, npos, ppg, block_table, seq_lens, tree_mask,
                    tree_start, sinks, window, scale, kps, ns, out, part_o, part_ml, ws.status)
        return
    kps, ns = split_plan(T, n_kv, max_len, num_sms, ws.max_splits)
    part_o = ws.part_o[: T * n_q * ns * d].view(T, n_q, ns, d)
    part_ml = ws.part_ml[: T * n_q * ns * 2].view(T, n_q, ns, 2)
    C().decode_attn(q, k_cache, v_cache, block_table, seq_lens, tree_mask, tree_start, sinks,
                    window, scale, softcap, kps, part_o, part_ml, out)
