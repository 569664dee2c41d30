"""LoRA adapters: loading, and per-request application on the GPU.

An adapter holds, per targeted weight (`blk.N.attn_q.weight`, ...), a pair
A [r, in] and B [out, r] and a scale alpha / r; the layer computes
W x + scale * B (A x).  Adapters come from llama.cpp-style LoRA GGUF files
(`<tensor>.lora_a` / `<tensor>.lora_b`, metadata `adapter.lora.alpha`) or
from tensors.

On the GPU a LoraSet stacks up to `max_adapters` adapters per fused target
of every layer (q|k|v, o, gate|up, down): A [M, R, in] and B [M, out, R] in
fp16 with the scale folded into B; the fused targets concatenate their parts'
ranks (A stacked, B block-diagonal).  Each token row carries an adapter index
(-1 = none), so requests with different adapters share a batch; the delta is
computed by the lora kernels and added by the GEMM's epilogue as it reads the
result (GemmOut.add).  The tables are allocated once (CUDA-graph safe); adding
an adapter fills a slot.

Reference: per-request LoRA from GGUF (src/inference/lora.rs, registry and
per-request adapter selection).
"""
from __future__ import annotations

import numpy as np
import torch

from ..gguf import quants as Q

# base tensor suffix -> (fused group, part index within the group)
_PARTS = {"attn_q": ("qkv", 0), "attn_k": ("qkv", 1), "attn_v": ("qkv", 2),
          "attn_output": ("o", 0), "ffn_gate": ("gu", 0), "ffn_up": ("gu", 1),
          "ffn_down": ("down", 0)}


class LoraAdapter:
    def __init__(self, name: str, alpha: float, tensors: dict):
        """tensors: base name (e.g. "blk.0.attn_q.weight") -> (A [r, in], B [out, r])."""
        self.name, self.alpha = name, float(alpha)
        self.tensors = {k: (np.asarray(a, np.float32), np.asarray(b, np.float32))
                        for k, (a, b) in tensors.items()}

    def scale(self, base: str) -> float:
        return self.alpha / self.tensors[base][0].shape[0]

    @classmethod
    def random(cls, cfg, rank: int = 8, seed: int = 0, alpha: float | None = None,
               std: float = 0.05, targets=tuple(_PARTS), layers=None,
               name: str | None = None) -> "LoraAdapter":
        """Random adapter of a model config (synthetic runs and tests)."""
        rng = np.random.default_rng(seed)
        d, H = cfg.head_dim, cfg.hidden
        qh = 2 * d if cfg.attn_output_gate else d
        dims = {"attn_q": (H, cfg.n_heads * qh), "attn_k": (H, cfg.n_kv_heads * d),
                "attn_v": (H, cfg.n_kv_heads * d), "attn_output": (cfg.n_heads * d, H),
                "ffn_gate": (H, cfg.ffn), "ffn_up": (H, cfg.ffn), "ffn_down": (cfg.ffn, H)}
        tensors = {}
        for i in (range(cfg.n_layers) if layers is None else layers):
            if cfg.is_linear_attn(i):
                continue
            for t in targets:
                k, n = dims[t]
                a = rng.standard_normal((rank, k)).astype(np.float32) / np.sqrt(k)
                b = rng.standard_normal((n, rank)).astype(np.float32) * std
                tensors[f"blk.{i}.{t}.weight"] = (a, b)
        return cls(name or f"random-{seed}", float(alpha if alpha is not None else rank), tensors)

    @classmethod
    def from_gguf(cls, path: str, name: str | None = None) -> "LoraAdapter":
        from ..gguf.file import GGUFReader
        r = GGUFReader(path)
        alpha = float(r.metadata.get("adapter.lora.alpha", 0.0))
        pairs: dict = {}
        for tname, ti in r.tensors.items():
            for suf, idx in ((".lora_a", 0), (".lora_b", 1)):
                if tname.endswith(suf):
                    base = tname[: -len(suf)]
                    arr = r.tensor_float(tname).reshape(ti.shape)
                    pairs.setdefault(base, [None, None])[idx] = arr
        tensors = {k: (v[0], v[1]) for k, v in pairs.items() if v[0] is not None and v[1] is not None}
        if not alpha and tensors:
            alpha = float(next(iter(tensors.values()))[0].shape[0])  # scale 1
        return cls(name or path, alpha, tensors)

    def write_gguf(self, path: str):
        from ..gguf.file import GGUFWriter
        w = GGUFWriter("llama")
        w.add("general.type", "adapter")
        w.add("adapter.type", "lora")
        w.add("adapter.lora.alpha", float(self.alpha))
        for base, (a, b) in self.tensors.items():
            w.add_tensor(base + ".lora_a", a.astype(np.float32), Q.F32, a.shape)
            w.add_tensor(base + ".lora_b", b.astype(np.float32), Q.F32, b.shape)
        w.write(path)


class LoraSet:
    """Stacked adapter tables of one LlamaGPU (layers lo..hi)."""

    def __init__(self, model, max_adapters: int = 4, max_rank: int = 64):
        self.model, self.M, self.R = model, max_adapters, max_rank
        self.names: list[str] = []
        self.tables: dict = {}   # (layer j, group) -> (A, B, scale)
        dev = model.device
        for j, L in enumerate(model.layers):
            for group, lin, n_parts in (("qkv", getattr(L, "wqkv", None), 3), ("o", getattr(L, "wo", None), 1),
                                        ("gu", getattr(L, "wgu", None), 2),
                                        ("down", getattr(L, "wdown", None), 1)):
                if lin is None:
                    continue
                R = max_rank * n_parts
                A = torch.zeros(max_adapters, R, lin.K, dtype=torch.float16, device=dev)
                B = torch.zeros(max_adapters, lin.rows, R, dtype=torch.float16, device=dev)
                S = torch.ones(max_adapters, dtype=torch.float32, device=dev)
                self.tables[(j, group)] = (A, B, S, n_parts)

    def index(self, name: str) -> int:
        return self.names.index(name)

    def remove(self, name: str) -> int:
        """Free an adapter's slot (its tables zeroed); returns the slot."""
        a = self.names.index(name)
        for At, Bt, S, _ in self.tables.values():
            At[a].zero_()
            Bt[a].zero_()
            S[a] = 1.0
        self.names[a] = None
        return a

    def add(self, ad: LoraAdapter) -> int:
        if ad.name in self.names:
            return self.names.index(ad.name)
        a = self.names.index(None) if None in self.names else len(self.names)
        if a >= self.M:
            raise ValueError(f"at most {self.M} adapters")
        cfg, m = self.model.cfg, self.model
        d = cfg.head_dim
        qh = 2 * d if cfg.attn_output_gate else d
        part_rows = {"qkv": [m.n_q * qh, m.n_kv * d, m.n_kv * d], "gu": [m.ffn_loc, m.ffn_loc]}
        for j, L in enumerate(m.layers):
            layer = m.lo + j
            for suffix, (group, part) in _PARTS.items():
                base = f"blk.{layer}.{suffix}.weight"
                if base not in ad.tensors or (j, group) not in self.tables:
                    continue
                A_, B_ = ad.tensors[base]
                r = A_.shape[0]
                if r > self.R:
                    raise ValueError(f"rank {r} > max_rank {self.R}")
                At, Bt, _, _ = self.tables[(j, group)]
                off = part * self.R
                rows = part_rows.get(group, [Bt.shape[1]])
                r0 = sum(rows[:part])
                At[a, off:off + r] = torch.from_numpy(A_).to(At.device, torch.float16)
                Bt[a, r0:r0 + B_.shape[0], off:off + r] = torch.from_numpy(
                    B_ * ad.scale(base)).to(Bt.device, torch.float16)
        if a == len(self.names):
            self.names.append(ad.name)
        else:
            self.names[a] = ad.name
        return a
