"""Block drafter (DFlash): a small model that guesses a whole block of tokens
in one forward from the target's own hidden states.

File (GGUF, architecture ``dflash``, llama.cpp's draft-dflash names):
  dflash.embedding_length, block_count, attention.head_count(_kv),
  attention.key_length, feed_forward_length, attention.layer_norm_rms_epsilon,
  rope.freq_base, block_size, target_layers (the target layers whose INPUT
  residual stream it reads, in order), attention.causal (optional),
  tokenizer.ggml.mask_token_id;
  fc.weight [H, len(target_layers) * H], enc.output_norm.weight, output_norm.weight,
  blk.{i}.attn_norm / attn_q / attn_k / attn_v / attn_output / attn_q_norm /
  attn_k_norm / ffn_norm / ffn_gate / ffn_up / ffn_down.

The computation (as the DFlash paper and the reference's
src/inference/split/block_drafter.rs describe it):
* context rows: the target's captured streams at each committed position,
  concatenated, through ``fc`` and ``enc.output_norm``; every drafter layer
  projects them (not through its input norm) into keys (k-normed, NEOX RoPE
  at their positions) and values, kept in the drafter's cache;
* a block [last token, mask x (B - 1)] at the next positions, embedded with
  the TARGET's token table; each layer: queries and keys/values from the
  normed block, the block attending to the whole context and to itself
  (both ways unless the file says causal), SwiGLU FFN, residuals;
* the output norm, then the TARGET's output head: row i >= 1 guesses the
  token at position start + i.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

from ..gguf import quants as Q

ARCH = "dflash"


@dataclass
class DFlashConfig:
    hidden: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    ffn: int
    block_size: int
    target_layers: tuple
    mask_token: int
    rms_eps: float = 1e-6
    rope_theta: float = 1e6
    causal: bool = False

    @staticmethod
    def from_metadata(md: dict) -> "DFlashConfig":
        g = lambda k, d=None: md.get(f"{ARCH}.{k}", d)
        H, nh = int(g("embedding_length")), int(g("attention.head_count"))
        return DFlashConfig(hidden=H, n_layers=int(g("block_count")), n_heads=nh,
                            n_kv_heads=int(g("attention.head_count_kv", nh)),
                            head_dim=int(g("attention.key_length", H // nh)),
                            ffn=int(g("feed_forward_length")), block_size=int(g("block_size", 16)),
                            target_layers=tuple(int(x) for x in g("target_layers")),
                            mask_token=int(md["tokenizer.ggml.mask_token_id"]),
                            rms_eps=float(g("attention.layer_norm_rms_epsilon", 1e-6)),
                            rope_theta=float(g("rope.freq_base", 1e6)),
                            causal=bool(g("attention.causal", False)))

    def metadata(self) -> dict:
        a = ARCH
        md = {"general.architecture": a, f"{a}.embedding_length": self.hidden,
              f"{a}.block_count": self.n_layers, f"{a}.attention.head_count": self.n_heads,
              f"{a}.attention.head_count_kv": self.n_kv_heads,
              f"{a}.attention.key_length": self.head_dim, f"{a}.feed_forward_length": self.ffn,
              f"{a}.attention.layer_norm_rms_epsilon": float(self.rms_eps),
              f"{a}.rope.freq_base": float(self.rope_theta), f"{a}.block_size": self.block_size,
              f"{a}.target_layers": [int(x) for x in self.target_layers],
              "tokenizer.ggml.mask_token_id": self.mask_token}
        if self.causal:
            md[f"{a}.attention.causal"] = True
        return md

    def tensor_specs(self, qtype: int) -> list:
        H, d, F = self.hidden, self.head_dim, self.ffn
        specs = [("fc.weight", (H, len(self.target_layers) * H), qtype),
                 ("enc.output_norm.weight", (H,), Q.F32), ("output_norm.weight", (H,), Q.F32)]
        for i in range(self.n_layers):
            b = f"blk.{i}."
            specs += [(b + "attn_norm.weight", (H,), Q.F32),
                      (b + "attn_q.weight", (self.n_heads * d, H), qtype),
                      (b + "attn_k.weight", (self.n_kv_heads * d, H), qtype),
                      (b + "attn_v.weight", (self.n_kv_heads * d, H), qtype),
                      (b + "attn_output.weight", (H, self.n_heads * d), qtype),
                      (b + "attn_q_norm.weight", (d,), Q.F32), (b + "attn_k_norm.weight", (d,), Q.F32),
                      (b + "ffn_norm.weight", (H,), Q.F32),
                      (b + "ffn_gate.weight", (F, H), qtype), (b + "ffn_up.weight", (F, H), qtype),
                      (b + "ffn_down.weight", (H, F), qtype)]
        return specs


def write_random_dflash(path: str, target_cfg, n_layers: int = 2, block_size: int = 8,
                        target_layers=None, mask_token: int | None = None, seed: int = 0,
                        qtype: str = "Q8_0", std: float = 0.02, causal: bool = False) -> DFlashConfig:
    """A random-init drafter for `target_cfg` (test models)."""
    from ..gguf.file import GGUFWriter
    n = target_cfg.n_layers
    tl = tuple(target_layers) if target_layers else tuple(sorted({1, max(1, n // 2), n}))
    dc = DFlashConfig(hidden=target_cfg.hidden, n_layers=n_layers, n_heads=target_cfg.n_heads,
                      n_kv_heads=target_cfg.n_kv_heads, head_dim=target_cfg.head_dim,
                      ffn=target_cfg.ffn or 4 * target_cfg.hidden, block_size=block_size,
                      target_layers=tl,
                      mask_token=target_cfg.vocab - 1 if mask_token is None else mask_token,
                      rope_theta=target_cfg.rope_theta, causal=causal)
    rng = np.random.default_rng(seed)
    w = GGUFWriter(ARCH)
    for k, v in dc.metadata().items():
        w.add(k, v)
    qt = Q.NAME_TO_TYPE[qtype]
    for name, shape, t in dc.tensor_specs(qt):
        if t == Q.F32:
            vals = np.ones(shape, np.float32)
        else:
            vals = rng.standard_normal(shape, dtype=np.float32) * std
        w.add_tensor(name, Q.quantize(vals.reshape(-1, shape[-1]), t), t, shape)
    w.write(path)
    return dc


def _rms(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


class DFlashDrafter:
    """A block drafter beside a CPU target model (LlamaCPU, last stage with
    the token table and output head)."""

    def __init__(self, path: str, target):
        from ..gguf.file import GGUFReader
        r = GGUFReader(path)
        if r.metadata.get("general.architecture") != ARCH:
            raise ValueError(f"{path} is not a {ARCH} drafter")
        dc = self.cfg = DFlashConfig.from_metadata(r.metadata)
        tc = target.cfg
        if dc.hidden != tc.hidden:
            raise ValueError("drafter and target widths differ")
        if not dc.target_layers or any(not 0 <= L <= tc.n_layers for L in dc.target_layers):
            raise ValueError(f"target layers {dc.target_layers} of a {tc.n_layers}-layer model")
        if not 0 <= dc.mask_token < tc.vocab or dc.block_size < 2:
            raise ValueError("mask token past the vocabulary, or a block under 2")
        if dc.n_heads % dc.n_kv_heads:
            raise ValueError("query heads do not share KV heads evenly")

        def get(name):
            ti = r.tensors[name]
            raw = np.array(r.tensor_bytes(name), copy=True).reshape(-1)
            return torch.from_numpy(Q.dequantize(raw, ti.qtype).reshape(ti.shape)).float()
        self.target = target
        self.fc, self.hidden_norm = get("fc.weight"), get("enc.output_norm.weight")
        self.out_norm = get("output_norm.weight")
        self.layers = []
        for i in range(dc.n_layers):
            b = f"blk.{i}."
            self.layers.append({k: get(b + k + ".weight") for k in (
                "attn_norm", "attn_q", "attn_k", "attn_v", "attn_output", "attn_q_norm",
                "attn_k_norm", "ffn_norm", "ffn_gate", "ffn_up", "ffn_down")})
        d = dc.head_dim
        self.inv_freq = 1.0 / (dc.rope_theta ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
        self.reset()

    def reset(self):
        """Forget the context (a new sequence)."""
        self.ctx_k = [None] * self.cfg.n_layers
        self.ctx_v = [None] * self.cfg.n_layers
        self.n_ctx = 0

    def _rope(self, x, pos):
        """NEOX rotation of x [n, heads, d] at positions pos [n]."""
        ang = pos.float()[:, None] * self.inv_freq[None, :]
        c, s = torch.cos(ang)[:, None, :], torch.sin(ang)[:, None, :]
        half = x.shape[-1] // 2
        a, b = x[..., :half], x[..., half:]
        return torch.cat([a * c - b * s, b * c + a * s], -1)

    def _kv(self, L, x, pos):
        dc = self.cfg
        n = x.shape[0]
        k = _rms((x @ L["attn_k"].T).view(n, dc.n_kv_heads, dc.head_dim), L["attn_k_norm"], dc.rms_eps)
        v = (x @ L["attn_v"].T).view(n, dc.n_kv_heads, dc.head_dim)
        return self._rope(k, pos), v

    def add_context(self, captured: dict, rows, positions: torch.Tensor):
        """Take in committed positions: the target's captured input streams of
        the target layers at `rows`, at `positions` (the next ones in order)."""
        dc = self.cfg
        feats = torch.cat([captured[L][rows].float() for L in dc.target_layers], -1)
        ctx = _rms(feats @ self.fc.T, self.hidden_norm, dc.rms_eps)
        for i, L in enumerate(self.layers):
            k, v = self._kv(L, ctx, positions)
            self.ctx_k[i] = k if self.ctx_k[i] is None else torch.cat([self.ctx_k[i], k])
            self.ctx_v[i] = v if self.ctx_v[i] is None else torch.cat([self.ctx_v[i], v])
        self.n_ctx += len(positions)

    def draft(self, last_token: int, start: int) -> list[int]:
        """The block [last_token, mask ...] at positions start.. through the
        drafter: the B - 1 guessed tokens for positions start+1 .. start+B-1."""
        dc, t = self.cfg, self.target
        B = dc.block_size
        toks = torch.tensor([last_token] + [dc.mask_token] * (B - 1))
        x = t.embd[toks].float()
        pos = torch.arange(start, start + B)
        rep = dc.n_heads // dc.n_kv_heads
        scale = 1.0 / math.sqrt(dc.head_dim)
        for i, L in enumerate(self.layers):
            xn = _rms(x, L["attn_norm"], dc.rms_eps)
            q = _rms((xn @ L["attn_q"].T).view(B, dc.n_heads, dc.head_dim), L["attn_q_norm"], dc.rms_eps)
            q = self._rope(q, pos)
            kb, vb = self._kv(L, xn, pos)
            K = kb if self.ctx_k[i] is None else torch.cat([self.ctx_k[i], kb])
            V = vb if self.ctx_v[i] is None else torch.cat([self.ctx_v[i], vb])
            Kr, Vr = K.repeat_interleave(rep, 1), V.repeat_interleave(rep, 1)
            s = torch.einsum("bhd,nhd->hbn", q, Kr) * scale
            if dc.causal:   # the block sees the context and its own earlier rows
                n_ctx = K.shape[0] - B
                j = torch.arange(K.shape[0])[None, :]
                allow = j < n_ctx + torch.arange(B)[:, None] + 1
                s = s.masked_fill(~allow[None], float("-inf"))
            a = torch.einsum("hbn,nhd->bhd", torch.softmax(s, -1), Vr).reshape(B, -1)
            x = x + a @ L["attn_output"].T
            xn = _rms(x, L["ffn_norm"], dc.rms_eps)
            x = x + (torch.nn.functional.silu(xn @ L["ffn_gate"].T) * (xn @ L["ffn_up"].T)) @ L["ffn_down"].T
        out = _rms(x, self.out_norm, dc.rms_eps)
        logits = t._logits(out[1:].to(t.dtype))
        return [int(v) for v in logits.argmax(-1)]
