"""Weight sources: where a model's tensors come from.

* ``GgufSource``     a GGUF file (mmap) or a shard directory (reference shard
                     layout), tensor bytes in GGML block format.
* ``RandomSource``   random-init weights of a given architecture, generated
                     directly in GGML block format -- on the GPU for the big
                     benchmark models (no 40 GB file to write), or on the host
                     (N(0, std) floats quantized exactly) for test models.

Tensor names follow the llama.cpp GGUF convention (``token_embd.weight``,
``blk.N.attn_q.weight``, ``blk.N.ffn_down.weight``, ``output.weight`` ...).
Every source returns ``(bytes, qtype, shape)`` with ``shape`` in numpy order.
"""
from __future__ import annotations

import hashlib

import numpy as np
import torch

from ..gguf import quants as Q
from ..gguf.file import GGUFReader, GGUFWriter, ShardedGguf
from .config import ModelConfig, from_gguf_metadata, to_gguf_metadata
from .layout import LAYOUT_FAMILIES, file_specs, kernel_name, to_file, to_kernel


def _layer_specs(cfg: ModelConfig, i: int, wq: int, xq: int) -> list:
    """(name, shape, qtype) of layer i's tensors."""
    H = cfg.hidden
    specs = []
    b = f"blk.{i}."
    specs.append((b + "attn_norm.weight", (H,), Q.F32))
    if cfg.is_linear_attn(i):
        nk, nv, dh = cfg.ssm_k_heads, cfg.ssm_v_heads, cfg.ssm_head_dim
        qkv = 2 * nk * dh + nv * dh
        specs += [(b + "attn_qkv.weight", (qkv, H), wq),
                  (b + "attn_gate.weight", (nv * dh, H), wq),
                  (b + "ssm_ba.weight", (2 * nv, H), Q.F32),
                  (b + "ssm_conv1d.weight", (qkv, cfg.ssm_conv_kernel), Q.F32),
                  (b + "ssm_dt.bias", (nv,), Q.F32),
                  (b + "ssm_a", (nv,), Q.F32),
                  (b + "ssm_norm.weight", (dh,), Q.F32),
                  (b + "ssm_out.weight", (H, nv * dh), wq)]
    else:
        qrows = cfg.q_dim * (2 if cfg.attn_output_gate else 1)
        if cfg.fused_qkv:
            specs.append((b + "attn_qkv.weight", (qrows + 2 * cfg.kv_dim, H), wq))
            if cfg.attn_bias:
                specs.append((b + "attn_qkv.bias", (qrows + 2 * cfg.kv_dim,), Q.F32))
        else:
            specs += [(b + "attn_q.weight", (qrows, H), wq),
                      (b + "attn_k.weight", (cfg.kv_dim, H), wq),
                      (b + "attn_v.weight", (cfg.kv_dim, H), wq)]
            if cfg.attn_bias:
                specs += [(b + "attn_q.bias", (cfg.q_dim,), Q.F32),
                          (b + "attn_k.bias", (cfg.kv_dim,), Q.F32),
                          (b + "attn_v.bias", (cfg.kv_dim,), Q.F32)]
        specs.append((b + "attn_output.weight", (H, cfg.q_dim), wq))
        if cfg.has_out_bias:
            specs.append((b + "attn_output.bias", (H,), Q.F32))
        if cfg.post_norms:
            specs.append((b + "post_attention_norm.weight", (H,), Q.F32))
        if cfg.qk_norm:
            specs += [(b + "attn_q_norm.weight", (cfg.head_dim,), Q.F32),
                      (b + "attn_k_norm.weight", (cfg.head_dim,), Q.F32)]
        if cfg.attn_sinks:
            specs.append((b + "attn_sinks.weight", (cfg.n_heads,), Q.F32))
    specs.append((b + "ffn_norm.weight", (H,), Q.F32))
    if cfg.is_moe_layer(i):
        E, F = cfg.n_experts, cfg.expert_ffn
        specs += [(b + "ffn_gate_inp.weight", (E, H), Q.F32),
                  (b + "ffn_gate_exps.weight", (E, F, H), xq),
                  (b + "ffn_up_exps.weight", (E, F, H), xq),
                  (b + "ffn_down_exps.weight", (E, H, F), xq)]
        if cfg.arch == "gpt-oss":
            specs += [(b + "ffn_gate_inp.bias", (E,), Q.F32),
                      (b + "ffn_gate_exps.bias", (E, F), Q.F32),
                      (b + "ffn_up_exps.bias", (E, F), Q.F32),
                      (b + "ffn_down_exps.bias", (E, H), Q.F32)]
        if cfg.moe_gating == "sigmoid" and cfg.moe_sel_bias:
            specs.append((b + "exp_probs_b.bias", (E,), Q.F32))
        if cfg.shared_expert_ffn:
            S = cfg.shared_expert_ffn
            specs += [(b + "ffn_gate_shexp.weight", (S, H), wq),
                      (b + "ffn_up_shexp.weight", (S, H), wq),
                      (b + "ffn_down_shexp.weight", (H, S), wq)]
            if cfg.shared_expert_gated:
                specs.append((b + "ffn_gate_inp_shexp.weight", (H,), Q.F32))
    elif cfg.fused_gate_up:
        specs += [(b + "ffn_up.weight", (2 * cfg.ffn, H), wq),
                  (b + "ffn_down.weight", (H, cfg.ffn), wq)]
    else:
        specs += [(b + "ffn_gate.weight", (cfg.ffn, H), wq),
                  (b + "ffn_up.weight", (cfg.ffn, H), wq),
                  (b + "ffn_down.weight", (H, cfg.ffn), wq)]
    if cfg.post_norms and not cfg.is_linear_attn(i):
        specs.append((b + "post_ffw_norm.weight", (H,), Q.F32))
    return specs


def tensor_specs(cfg: ModelConfig) -> list[tuple[str, tuple, int]]:
    """(name, shape, qtype) of every tensor of a model (llama.cpp names)."""
    wq = Q.NAME_TO_TYPE[cfg.weight_qtype]
    eq = Q.NAME_TO_TYPE[cfg.embed_qtype]
    oq = Q.NAME_TO_TYPE[cfg.output_qtype or cfg.weight_qtype]
    xq = Q.NAME_TO_TYPE[cfg.expert_qtype or cfg.weight_qtype]
    H = cfg.hidden
    specs = [("token_embd.weight", (cfg.vocab, H), eq)]
    for i in range(cfg.n_layers):
        specs += _layer_specs(cfg, i, wq, xq)
    for i in range(cfg.n_layers, cfg.n_layers + cfg.mtp_layers):
        # a next-token-prediction block: a full-attention layer whose input is
        # eh_proj([enorm(embedding of the next token) | hnorm(trunk hidden)])
        b = f"blk.{i}."
        specs += _layer_specs(cfg, i, wq, xq)
        specs += [(b + "nextn.eh_proj.weight", (H, 2 * H), wq),
                  (b + "nextn.enorm.weight", (H,), Q.F32),
                  (b + "nextn.hnorm.weight", (H,), Q.F32),
                  (b + "nextn.shared_head_norm.weight", (H,), Q.F32)]
    specs.append(("output_norm.weight", (H,), Q.F32))
    if not cfg.tie_embeddings:
        specs.append(("output.weight", (cfg.vocab, H), oq))
    if cfg.quant_mix:
        mixed = []
        for name, shape, qt in specs:
            layer, base = -1, name
            if name.startswith("blk."):
                _, num, base = name.split(".", 2)
                layer = int(num)
            t = cfg.tensor_qtype(base, layer)
            mixed.append((name, shape, Q.NAME_TO_TYPE[t] if t and len(shape) == 2 else qt))
        specs = mixed
    return specs


def _is_norm(name: str) -> bool:
    return name.endswith("norm.weight") or name.endswith("norm.weight.post")


def _init_value(name: str, shape, rng: np.random.Generator, std: float) -> np.ndarray:
    if _is_norm(name):
        return np.ones(shape, np.float32)
    if name.endswith("ssm_a"):
        return -np.exp(rng.uniform(0, 1, shape)).astype(np.float32)
    if name.endswith("ssm_dt.bias"):
        return rng.uniform(-1, 1, shape).astype(np.float32)
    if name.endswith("attn_sinks.weight"):
        return rng.standard_normal(shape).astype(np.float32)
    if name.endswith("exp_probs_b.bias"):
        return rng.uniform(-0.05, 0.05, shape).astype(np.float32)
    if name.endswith("ffn_gate_inp.weight"):
        # routers: peaked top-k (logit std ~ 5) like trained routers, not near-uniform
        return (rng.standard_normal(shape, dtype=np.float32) * (5.0 / np.sqrt(shape[-1]))).astype(np.float32)
    return (rng.standard_normal(shape, dtype=np.float32) * std).astype(np.float32)


class GgufSource:
    def __init__(self, path: str, layers: tuple[int, int] | None = None):
        import os
        if os.path.isdir(path):
            self.f = ShardedGguf(path, layers=layers)
        else:
            self.f = GGUFReader(path)
        self.cfg = from_gguf_metadata(self.f.metadata)
        if self.cfg.arch == "glm4moe" and "swarmllm.config" not in self.f.metadata:
            # GLM-4.5 files say whether they carry q/k norms by the tensors alone
            self.cfg.qk_norm = "blk.0.attn_q_norm.weight" in self.f.tensors
        # per-pair frequency divisors stored as tensors: Llama 3.1-3.3 files
        # carry their llama3 scaling as rope_freqs (each pair's angle divided
        # by its factor; reference: split/loader/mod.rs load_rope_freqs);
        # LongRoPE (phi3) as short / long factors, the short ones serving
        # contexts up to the original training length
        for name in ("rope_freqs.weight", "rope_factors_short.weight", "rope_factors_long.weight"):
            if self.cfg.rope_factors is None and name in self.f.tensors:
                t, qt, shape = self.get(name)
                self.cfg.rope_factors = Q.dequantize(t.numpy().reshape(-1), qt).tolist()

    def has(self, name: str) -> bool:
        return all(n in self.f.tensors for n in kernel_name(self.cfg.arch, name))

    def _raw(self, name: str):
        ti = self.f.tensors[name]
        return np.array(self.f.tensor_bytes(name), copy=True).reshape(-1), ti.qtype, ti.shape

    def get(self, name: str, device=None):
        """A tensor as (bytes, qtype, shape), in the kernels' order: the hybrid
        families' DeltaNet tensors are reordered from the file's (layout.py)."""
        if self.cfg.arch in LAYOUT_FAMILIES:
            raw, qt, shape = to_kernel(self.cfg, name, self._raw)
        else:
            raw, qt, shape = self._raw(name)
        t = torch.from_numpy(np.ascontiguousarray(raw))
        if device is not None:
            t = t.to(device)
        return t, qt, shape


class RandomSource:
    """Deterministic random-init weights.  `device=cuda` tensors of quantized
    types are produced directly as random GGML blocks on the GPU (values
    roughly N(0, std)); host tensors are N(0, std) floats quantized exactly."""

    def __init__(self, cfg: ModelConfig, seed: int = 0, std: float = 0.02, on_device: bool = False):
        self.cfg, self.seed, self.std, self.on_device = cfg, seed, std, on_device
        self.specs = {n: (s, q) for n, s, q in tensor_specs(cfg)}

    def has(self, name: str) -> bool:
        return name in self.specs

    def _rng(self, name: str) -> np.random.Generator:
        h = int.from_bytes(hashlib.sha256(f"{self.seed}:{name}".encode()).digest()[:8], "little")
        return np.random.default_rng(h)

    def get(self, name: str, device=None):
        shape, qt = self.specs[name]
        n = int(np.prod(shape))
        dev_ok = device is not None and torch.device(device).type == "cuda"
        if self.on_device and dev_ok and qt in (Q.Q4_K, Q.Q6_K, Q.Q8_0, Q.F16, Q.BF16, Q.MXFP4) \
                and not _is_norm(name):
            return _random_blocks_device(name, shape, qt, self.seed, self.std, device), qt, shape
        vals = _init_value(name, shape, self._rng(name), self.std)
        b = Q.quantize(vals.reshape(-1, shape[-1]), qt)
        t = torch.from_numpy(np.ascontiguousarray(b).reshape(-1))
        if device is not None:
            t = t.to(device)
        assert t.numel() == Q.nbytes(qt, n)
        return t, qt, shape


def _random_blocks_device(name, shape, qt, seed, std, device) -> torch.Tensor:
    """Random GGML blocks generated on the device (uint8, flat)."""
    h = int.from_bytes(hashlib.sha256(f"{seed}:{name}".encode()).digest()[:8], "little")
    g = torch.Generator(device=device)
    g.manual_seed(h & ((1 << 63) - 1))
    n = int(np.prod(shape))
    if qt in (Q.F16, Q.BF16):
        dt = torch.float16 if qt == Q.F16 else torch.bfloat16
        return (torch.randn(n, generator=g, device=device) * std).to(dt).view(torch.uint8)
    if qt == Q.MXFP4:
        nb = n // 32
        out = torch.empty(nb, 17, dtype=torch.uint8, device=device)
        # |code| up to 12 -> choose e so that 12*2^(e-128) ~ 3 std
        e = int(round(np.log2(3 * std / 12.0))) + 128
        out[:, 0] = e
        out[:, 1:] = torch.randint(0, 256, (nb, 16), generator=g, device=device, dtype=torch.int32).to(torch.uint8)
        return out.reshape(-1)
    if qt == Q.Q6_K:
        # codes q - 32 uniform in [-32, 31] (std 18.5); scales 30..63 (mean 46.5)
        nb = n // 256
        out = torch.empty(nb, 210, dtype=torch.uint8, device=device)
        out[:, :192] = torch.randint(0, 256, (nb, 192), generator=g, device=device,
                                     dtype=torch.int32).to(torch.uint8)
        out[:, 192:208] = torch.randint(30, 64, (nb, 16), generator=g, device=device,
                                        dtype=torch.int32).to(torch.uint8)
        d = torch.full((nb,), std / (18.5 * 46.5), device=device, dtype=torch.float16)
        out[:, 208:210] = d.view(torch.uint8).view(nb, 2)
        return out.reshape(-1)
    if qt == Q.Q8_0:
        # int8 codes uniform in [-128, 127] (std 73.9)
        nb = n // 32
        out = torch.empty(nb, 34, dtype=torch.uint8, device=device)
        d = torch.full((nb,), std / 73.9, device=device, dtype=torch.float16)
        out[:, 0:2] = d.view(torch.uint8).view(nb, 2)
        out[:, 2:] = torch.randint(0, 256, (nb, 32), generator=g, device=device,
                                   dtype=torch.int32).to(torch.uint8)
        return out.reshape(-1)
    assert qt == Q.Q4_K
    nb = n // 256
    out = torch.empty(nb, 144, dtype=torch.uint8, device=device)
    sc = torch.randint(40, 64, (nb, 8), generator=g, device=device, dtype=torch.int32)
    m = torch.randint(40, 64, (nb, 8), generator=g, device=device, dtype=torch.int32)
    # uniform codes 0..15 have std 4.61; per-code step s gives std ~ 4.61 s
    s = std / 4.61
    d = torch.full((nb,), s / 51.5, device=device, dtype=torch.float16)
    dmin = torch.full((nb,), 7.5 * s / 51.5, device=device, dtype=torch.float16)
    out[:, 0:2] = d.view(torch.uint8).view(nb, 2)
    out[:, 2:4] = dmin.view(torch.uint8).view(nb, 2)
    s12 = torch.zeros(nb, 12, dtype=torch.int32, device=device)
    for j in range(4):
        s12[:, j] = (sc[:, j] & 63) | ((sc[:, j + 4] >> 4) << 6)
        s12[:, j + 4] = (m[:, j] & 63) | ((m[:, j + 4] >> 4) << 6)
        s12[:, j + 8] = (sc[:, j + 4] & 0xF) | ((m[:, j + 4] & 0xF) << 4)
    out[:, 4:16] = s12.to(torch.uint8)
    out[:, 16:] = torch.randint(0, 256, (nb, 128), generator=g, device=device, dtype=torch.int32).to(torch.uint8)
    return out.reshape(-1)


def write_random_gguf(cfg: ModelConfig, path: str, seed: int = 0, std: float = 0.02):
    """Write a complete random-init GGUF (host generation; for test-size models)."""
    src = RandomSource(cfg, seed=seed, std=std)
    w = GGUFWriter(cfg.arch)
    for k, v in to_gguf_metadata(cfg).items():
        w.add(k, v)
    for name, shape, qt in file_specs(cfg, tensor_specs(cfg)):
        data = to_file(cfg, name, shape, qt, lambda n: src.get(n)[0].numpy())
        w.add_tensor(name, data, qt, shape)
    w.write(path)
    return path
