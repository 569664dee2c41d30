"""Model architecture configs, the benchmark presets, and GGUF metadata mapping.

Families (reference: ``src/inference/model_arch.rs:7-67``, architecture
mapping in ``src/inference/split/loader/mod.rs``):

* ``llama``     dense decoder: GQA attention, SwiGLU FFN, RMSNorm, RoPE
                (GGML "norm" interleaved pairs), optional llama3 / linear /
                YaRN frequency scaling.
* ``gpt-oss``   MoE decoder: attention with learned sinks and bias, sliding
                window on alternate layers, YaRN RoPE (NEOX), top-k softmax
                routed experts with clamped SwiGLU, MXFP4 experts.
* ``qwen3next`` hybrid: gated DeltaNet linear-attention layers and gated full
                attention layers (3:1), q/k RMSNorm, partial NEOX RoPE,
                512-expert MoE with a shared expert.
* ``qwen35`` / ``qwen35moe``  Qwen 3.5: the same hybrid layers with a dense
                SwiGLU FFN (``qwen35``) or routed experts plus a shared expert
                (``qwen35moe``); its files tile the value heads over the key
                heads and keep beta and alpha apart, which the loader puts in
                the kernels' order (models/layout.py).

The other families are the dense / MoE decoder with options, read from the
GGUF architecture name (llama.cpp's names and metadata keys):

* ``mistral``   Llama layout.
* ``qwen2``     q/k/v biases, NEOX RoPE (Qwen2 / Qwen2.5).
* ``qwen3``     per-head q/k RMSNorm, NEOX RoPE.
* ``qwen2moe``  Qwen2 attention; softmax over all experts, top-k without
                renormalisation, sigmoid-gated shared expert.
* ``qwen3moe``  Qwen3 attention; top-k then softmax over the selected experts.
* ``gemma``     GELU(tanh)-gated FFN, embeddings scaled by sqrt(hidden), tied
                output, NEOX RoPE.
* ``gemma2``    Gemma plus post-attention / post-FFN norms on each branch,
                attention-logit and final-logit soft-capping, a sliding window
                on every other layer.
* ``gemma3``    Gemma 2's layout with q/k RMSNorm, no soft-capping, five
                windowed layers to each global one, and RoPE base 10000 on the
                windowed layers.
* ``phi3``      fused q|k|v and gate|up tensors, NEOX RoPE, optional
                LongRoPE per-dimension factors.
* ``glm4``      fused q|k|v with biases, fused gate|up, partial interleaved
                RoPE, post-attention / post-FFN norms.
* ``glm4moe``   GLM-4.5: q/k/v with biases, partial NEOX RoPE, optional q/k
                norms, leading dense layers, then sigmoid-scored experts chosen
                with a selection bias (``exp_probs_b``), renormalised and
                scaled, plus an ungated shared expert; the file's
                ``post_attention_norm`` is the norm before the FFN; the
                trailing next-token-prediction blocks are not run.
* ``llama4``    Llama 4 (Scout / Maverick): interleaved RoPE with every 4th
                layer NoPE, per-head q/k RMS normalisation without a weight
                on the RoPE layers, sigmoid-scored experts whose weight
                scales the expert's input, an ungated shared expert, dense
                and routed layers interleaved (``interleave_moe_layer_step``).
                Runs on the CPU model; the GPU model refuses it by name.
* ``granite``   Llama with four multipliers (embedding, residual, attention,
                logit).  The GPU model runs files whose residual multiplier is
                1 (the others map to options it has); the CPU model runs all.
* ``qwen2vl`` / ``qwen3vl`` files: their text trunk is read as ``qwen2`` /
  ``qwen3``.
"""
from __future__ import annotations

import math
from dataclasses import asdict, dataclass, field, replace

import numpy as np


@dataclass
class ModelConfig:
    name: str = "model"
    arch: str = "llama"
    n_layers: int = 2
    hidden: int = 256
    n_heads: int = 4
    n_kv_heads: int = 2
    head_dim: int = 64
    ffn: int = 512
    vocab: int = 32000
    rope_theta: float = 10000.0
    rope_scaling: dict | None = None    # {"type": "llama3"|"yarn"|"linear", ...}
    rope_neox: bool = False             # False = GGML "norm" interleaved pairs
    rope_dim: int = 0                   # 0 -> head_dim (partial rotary otherwise)
    rms_eps: float = 1e-5
    tie_embeddings: bool = False
    attn_bias: bool = False
    qk_norm: bool = False
    attn_sinks: bool = False
    sliding_window: int = 0
    swa_every: int = 0                  # layer l uses SWA if swa_every and l % swa_every == 0
    attn_output_gate: bool = False      # qwen3next gated attention
    attn_out_bias: bool | None = None   # output-projection bias (None: same as attn_bias)
    act: str = "silu"                   # gated-FFN activation: "silu" | "gelu" (tanh approximation)
    embed_scale: float = 0.0            # token embeddings times this (0: none; gemma sqrt(hidden))
    attn_softcap: float = 0.0           # attention logits c * tanh(s / c) (gemma2)
    final_softcap: float = 0.0          # output logits c * tanh(l / c) (gemma2)
    post_norms: bool = False            # RMSNorm of each branch output before the residual add
    swa_pattern: int = 0                # layer l windowed iff (l + 1) % swa_pattern != 0 (gemma3)
    rope_local_theta: float = 0.0       # RoPE base of the windowed layers (gemma3), 0: same
    attn_scale: float = 0.0             # softmax scale (0: 1 / sqrt(head_dim))
    fused_qkv: bool = False             # file layout: one attn_qkv tensor (phi3, glm4)
    fused_gate_up: bool = False         # file layout: ffn_up holds gate | up (phi3, glm4)
    rope_factors: list | None = None    # LongRoPE per-pair frequency divisors (phi3)
    # MoE
    n_experts: int = 0
    n_experts_used: int = 0
    expert_ffn: int = 0
    shared_expert_ffn: int = 0
    moe_softmax_after_topk: bool = True  # gpt-oss: softmax over the selected logits
    moe_gating: str = "softmax"         # "sigmoid": GLM-4.5 scores with a selection bias
    moe_norm_topk: bool = True          # sigmoid gating: weights divided by their sum
    moe_scale: float = 1.0              # sigmoid gating: routed-weight multiplier
    moe_dense_layers: int = 0           # leading layers with a dense FFN (size `ffn`)
    moe_every: int = 0                  # > 1: only every Nth layer (1-based) routes (llama4 interleave)
    moe_sel_bias: bool = True           # sigmoid gating: the file has an exp_probs_b selection bias
    moe_weight_input: bool = False      # routed weight scales the expert's input, not its output (llama4)
    nope_every: int = 0                 # every Nth layer (1-based) has no RoPE (llama4 iRoPE)
    qk_rms_plain: bool = False          # q/k RMS-normalised per head without a weight on RoPE layers (llama4)
    residual_scale: float = 0.0         # branch outputs times this before the residual add (granite; 0: none)
    logit_scale: float = 0.0            # output logits divided by this (granite; 0: none)
    shared_expert_gated: bool = True    # a sigmoid gate (ffn_gate_inp_shexp) on the shared expert
    mtp_layers: int = 0                 # next-token-prediction blocks after the trunk (blk.{n_layers})
    swiglu_limit: float = 0.0           # gpt-oss clamped SwiGLU (7.0)
    swiglu_alpha: float = 1.702
    # hybrid linear attention (gated DeltaNet)
    full_attn_interval: int = 0         # every Nth layer (1-based) is full attention
    ssm_k_heads: int = 0
    ssm_v_heads: int = 0
    ssm_head_dim: int = 128
    ssm_conv_kernel: int = 4
    # storage types
    weight_qtype: str = "Q4_K"
    embed_qtype: str = "F16"
    output_qtype: str = ""              # "" -> weight_qtype
    expert_qtype: str = ""              # "" -> weight_qtype
    # per-tensor mix on top of weight_qtype: "q4_k_m" = Q6_K for the LM head and
    # for attn_v / ffn_down of the layers more_bits_layer() picks
    quant_mix: str = ""

    @property
    def q_dim(self) -> int:
        return self.n_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    @property
    def rot_dim(self) -> int:
        return self.rope_dim or self.head_dim

    def is_swa(self, layer: int) -> bool:
        if not self.sliding_window or self.is_mtp_block(layer):   # MTP blocks attend fully
            return False
        if self.swa_pattern:
            return (layer + 1) % self.swa_pattern != 0
        return bool(self.swa_every and layer % self.swa_every == 0)

    @property
    def has_out_bias(self) -> bool:
        return self.attn_bias if self.attn_out_bias is None else self.attn_out_bias

    @property
    def softmax_scale(self) -> float:
        return self.attn_scale or 1.0 / math.sqrt(self.head_dim)

    def more_bits_layer(self, layer: int) -> bool:
        """Layers a "k_m" mix stores at higher precision: the first and last
        eighth of the stack and every third layer between them (the layers
        whose quantization error costs the most perplexity)."""
        n, e = self.n_layers, self.n_layers // 8
        return layer < e or layer >= n - e or (layer - e) % 3 == 2

    def tensor_qtype(self, name: str, layer: int = -1) -> str | None:
        """Storage type the quant mix gives `name` (None: the default rule)."""
        if self.quant_mix != "q4_k_m":
            return None
        if name == "output.weight":
            return "Q6_K"
        if name in ("attn_v.weight", "ffn_down.weight") and self.more_bits_layer(layer):
            return "Q6_K"
        return None

    def is_moe_layer(self, layer: int) -> bool:
        if not self.n_experts or layer < self.moe_dense_layers:
            return False
        return self.moe_every <= 1 or (layer + 1) % self.moe_every == 0

    def is_nope(self, layer: int) -> bool:
        """A layer without rotary position embedding (llama4: every 4th)."""
        return bool(self.nope_every) and (layer + 1) % self.nope_every == 0

    @property
    def moe_mode(self) -> int:
        """Routing mode of the top-k kernel: 0 softmax over all experts, 1
        top-k then softmax, 2 sigmoid scores with a selection bias."""
        if self.moe_gating == "sigmoid":
            return 2
        return 1 if self.moe_softmax_after_topk else 0

    def is_mtp_block(self, layer: int) -> bool:
        """A next-token-prediction block (after the trunk): full attention."""
        return self.mtp_layers > 0 and layer >= self.n_layers

    def is_linear_attn(self, layer: int) -> bool:
        return (bool(self.full_attn_interval) and not self.is_mtp_block(layer)
                and (layer + 1) % self.full_attn_interval != 0)

    def is_moe(self, layer: int) -> bool:
        return self.n_experts > 0

    def to_dict(self) -> dict:
        return asdict(self)

    def scaled(self, **kw) -> "ModelConfig":
        return replace(self, **kw)

    def param_count(self) -> int:
        h, L = self.hidden, self.n_layers
        attn = h * (self.q_dim + 2 * self.kv_dim) + self.q_dim * h
        if self.n_experts:
            ffn = self.n_experts * 3 * h * self.expert_ffn + h * self.n_experts
            ffn += 3 * h * self.shared_expert_ffn
        else:
            ffn = 3 * h * self.ffn
        emb = self.vocab * h * (1 if self.tie_embeddings else 2)
        return L * (attn + ffn) + emb


def rope_inv_freq(cfg: ModelConfig, local: bool = False) -> tuple[np.ndarray, float]:
    """Per-pair inverse frequencies (length rot_dim/2) and the cos/sin
    attention factor, including llama3 / linear / YaRN / LongRoPE scaling.
    The scaling rules are the published ones (Meta's llama3 rope_scaling;
    YaRN, Peng et al. 2023; LongRoPE, Ding et al. 2024); the reference
    implements the same in src/inference/split/rope.rs:66-249.  `local`: the
    windowed layers of a model with a separate local base (gemma3), which
    take no scaling."""
    d = cfg.rot_dim
    theta = cfg.rope_local_theta if (local and cfg.rope_local_theta) else cfg.rope_theta
    inv = 1.0 / (theta ** (np.arange(0, d, 2, dtype=np.float64) / d))
    factor_attn = 1.0
    rs = {} if (local and cfg.rope_local_theta) else (cfg.rope_scaling or {})
    t = rs.get("type")
    if cfg.rope_factors is not None and not (local and cfg.rope_local_theta):
        inv = inv / np.asarray(cfg.rope_factors, np.float64)[: d // 2]
        if t == "longrope":
            scale = rs.get("factor", 1.0)
            old = rs.get("original_max_position_embeddings", 4096)
            factor_attn = rs.get("attn_factor") or (
                math.sqrt(1 + math.log(scale) / math.log(old)) if scale > 1 else 1.0)
    if t == "linear":
        inv = inv / rs["factor"]
    elif t == "llama3":
        factor = rs.get("factor", 8.0)
        lo, hi = rs.get("low_freq_factor", 1.0), rs.get("high_freq_factor", 4.0)
        old = rs.get("original_max_position_embeddings", 8192)
        lo_wl, hi_wl = old / lo, old / hi
        wl = 2 * math.pi / inv
        smooth = (old / wl - lo) / (hi - lo)
        scaled = np.where(wl > lo_wl, inv / factor, inv)
        mid = (wl <= lo_wl) & (wl >= hi_wl)
        scaled = np.where(mid, (1 - smooth) * inv / factor + smooth * inv, scaled)
        inv = scaled
    elif t == "yarn":
        factor = rs.get("factor", 32.0)
        old = rs.get("original_max_position_embeddings", 4096)
        beta_fast, beta_slow = rs.get("beta_fast", 32.0), rs.get("beta_slow", 1.0)

        def corr_dim(rot):
            return d * math.log(old / (rot * 2 * math.pi)) / (2 * math.log(cfg.rope_theta))

        low = max(math.floor(corr_dim(beta_fast)), 0)
        high = min(math.ceil(corr_dim(beta_slow)), d - 1)
        ramp = np.clip((np.arange(d // 2, dtype=np.float64) - low) / max(high - low, 1e-3), 0, 1)
        extra = 1.0 - ramp  # 1 -> keep original (high frequency)
        inv = inv / factor * (1 - extra) + inv * extra
        factor_attn = 0.1 * math.log(factor) + 1.0
    return inv.astype(np.float32), float(factor_attn)


# --------------------------------------------------------------------------- presets
def tiny_llama() -> ModelConfig:
    """Tiny Llama for the two-CPU-peer split: 2 layers, hidden 256, 4/2 heads, d 64, FFN 512, Q4_0."""
    return ModelConfig(name="tiny-llama", arch="llama", n_layers=2, hidden=256, n_heads=4,
                       n_kv_heads=2, head_dim=64, ffn=512, vocab=32000, rope_theta=10000.0,
                       rms_eps=1e-5, weight_qtype="Q4_0", embed_qtype="Q4_0",
                       output_qtype="Q4_0")


def llama32_3b() -> ModelConfig:
    """Llama-3.2-3B architecture, Q4_K weights (single-GPU serving config)."""
    return ModelConfig(name="llama-3.2-3b", arch="llama", n_layers=28, hidden=3072, n_heads=24,
                       n_kv_heads=8, head_dim=128, ffn=8192, vocab=128256, rope_theta=500000.0,
                       rope_scaling={"type": "llama3", "factor": 32.0, "low_freq_factor": 1.0,
                                     "high_freq_factor": 4.0,
                                     "original_max_position_embeddings": 8192},
                       rms_eps=1e-5, tie_embeddings=True, weight_qtype="Q4_K", embed_qtype="F16",
                       output_qtype="Q4_K")


def llama32_1b() -> ModelConfig:
    """Drafter for config 3: Llama-3.2-1B architecture."""
    return ModelConfig(name="llama-3.2-1b", arch="llama", n_layers=16, hidden=2048, n_heads=32,
                       n_kv_heads=8, head_dim=64, ffn=8192, vocab=128256, rope_theta=500000.0,
                       rope_scaling={"type": "llama3", "factor": 32.0, "low_freq_factor": 1.0,
                                     "high_freq_factor": 4.0,
                                     "original_max_position_embeddings": 8192},
                       rms_eps=1e-5, tie_embeddings=True, weight_qtype="Q4_K", embed_qtype="F16",
                       output_qtype="Q4_K")


def llama33_70b() -> ModelConfig:
    """Llama-3.3-70B architecture, Q4_K (the headline benchmark model)."""
    return ModelConfig(name="llama-3.3-70b", arch="llama", n_layers=80, hidden=8192, n_heads=64,
                       n_kv_heads=8, head_dim=128, ffn=28672, vocab=128256, rope_theta=500000.0,
                       rope_scaling={"type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                                     "high_freq_factor": 4.0,
                                     "original_max_position_embeddings": 8192},
                       rms_eps=1e-5, weight_qtype="Q4_K", embed_qtype="F16", output_qtype="Q4_K")


def llama33_70b_q4km() -> ModelConfig:
    """Llama-3.3-70B with a Q4_K_M-like tensor mix: Q4_K weights, a Q6_K LM head,
    Q6_K attn_v / ffn_down on the more_bits_layer() layers."""
    cfg = llama33_70b()
    cfg.name, cfg.quant_mix, cfg.output_qtype = "llama-3.3-70b-q4km", "q4_k_m", "Q6_K"
    return cfg


def gpt_oss_120b_style() -> ModelConfig:
    """gpt-oss-120B-style MoE (MXFP4 experts, bf16 attention; expert-parallel config)."""
    return ModelConfig(name="gpt-oss-120b-style", arch="gpt-oss", n_layers=36, hidden=2880,
                       n_heads=64, n_kv_heads=8, head_dim=64, ffn=2880, vocab=201088,
                       rope_theta=150000.0, rope_neox=True,
                       rope_scaling={"type": "yarn", "factor": 32.0,
                                     "original_max_position_embeddings": 4096,
                                     "beta_fast": 32.0, "beta_slow": 1.0},
                       rms_eps=1e-5, attn_bias=True, attn_sinks=True, sliding_window=128,
                       swa_every=2, n_experts=128, n_experts_used=4, expert_ffn=2880,
                       swiglu_limit=7.0, swiglu_alpha=1.702, weight_qtype="BF16",
                       embed_qtype="BF16", output_qtype="BF16", expert_qtype="MXFP4")


def qwen3_next_80b_style() -> ModelConfig:
    """Qwen3-Next-80B-A3B-style hybrid (3 DeltaNet : 1 gated attention; long-prefill config)."""
    return ModelConfig(name="qwen3-next-80b-a3b-style", arch="qwen3next", n_layers=48,
                       hidden=2048, n_heads=16, n_kv_heads=2, head_dim=256, ffn=512,
                       vocab=151936, rope_theta=10000000.0, rope_neox=True, rope_dim=64,
                       rms_eps=1e-6, qk_norm=True, attn_output_gate=True, n_experts=512,
                       n_experts_used=10, expert_ffn=512, shared_expert_ffn=512,
                       moe_softmax_after_topk=False, full_attn_interval=4, ssm_k_heads=16,
                       ssm_v_heads=32, ssm_head_dim=128, ssm_conv_kernel=4, weight_qtype="Q4_K",
                       embed_qtype="F16", output_qtype="Q4_K", expert_qtype="Q4_K")


PRESETS = {
    "tiny-llama": tiny_llama,
    "llama-3.2-3b": llama32_3b,
    "llama-3.2-1b": llama32_1b,
    "llama-3.3-70b": llama33_70b,
    "llama-3.3-70b-q4km": llama33_70b_q4km,
    "gpt-oss-120b-style": gpt_oss_120b_style,
    "qwen3-next-80b-a3b-style": qwen3_next_80b_style,
}


def preset(name: str) -> ModelConfig:
    return PRESETS[name]()


# --------------------------------------------------------------------------- GGUF mapping
_FAMILIES = ("llama", "mistral", "qwen2", "qwen3", "qwen2moe", "qwen3moe", "gemma", "gemma2",
             "gemma3", "phi3", "glm4", "glm4moe", "gpt-oss", "qwen3next", "qwen35", "qwen35moe",
             "llama4", "granite")
_ARCH_KEYS = {f: f for f in _FAMILIES}    # GGUF general.architecture == family name
# Architecture names whose language model is another family's, tensor for
# tensor: the Qwen2.5-VL / Qwen3-VL text trunks (their multimodal position
# sections turn a text-only position as NEOX RoPE does; image inputs are the
# vision encoder's business).  Reference: src/inference/model_arch.rs:84-99.
_ARCH_ALIASES = {"qwen2vl": "qwen2", "qwen3vl": "qwen3"}


def apply_family(cfg: ModelConfig, md: dict | None = None, prefix: str | None = None) -> ModelConfig:
    """Set the options a family implies (and those its GGUF metadata carries,
    under the keys of `prefix`, the file's architecture name)."""
    fam = cfg.arch
    pre = prefix or fam
    g = (lambda k, d=None: md.get(f"{pre}.{k}", d)) if md is not None else (lambda k, d=None: d)
    if fam in ("qwen2", "qwen2moe"):
        cfg.rope_neox, cfg.attn_bias, cfg.attn_out_bias = True, True, False
    if fam in ("qwen3", "qwen3moe"):
        cfg.rope_neox, cfg.qk_norm = True, True
    if fam == "qwen2moe":
        cfg.moe_softmax_after_topk = False      # softmax over all experts, no renormalisation
    if fam in ("gemma", "gemma2", "gemma3"):
        cfg.rope_neox, cfg.act, cfg.tie_embeddings = True, "gelu", True
        cfg.embed_scale = math.sqrt(cfg.hidden)
    if fam == "gemma2":
        cfg.post_norms, cfg.swa_every = True, 2
        cfg.attn_softcap = float(g("attn_logit_softcapping", cfg.attn_softcap or 50.0))
        cfg.final_softcap = float(g("final_logit_softcapping", cfg.final_softcap or 30.0))
    if fam == "gemma3":
        cfg.post_norms, cfg.qk_norm, cfg.swa_pattern = True, True, 6
        cfg.rope_local_theta = cfg.rope_local_theta or 10000.0
    if md is not None and not cfg.attn_scale and (fam, cfg.n_layers) in (("gemma2", 46),
                                                                      ("gemma3", 62)):
        # the 27B members scale queries by 1/sqrt(hidden / heads), not
        # 1/sqrt(head_dim) (query_pre_attn_scalar; the width in integers, as
        # llama.cpp computes it).  Reference: split/gguf_meta.rs:570 query_scale.
        width = cfg.hidden // cfg.n_heads
        if width != cfg.head_dim and width > 0:
            cfg.attn_scale = 1.0 / math.sqrt(width)
    if fam == "phi3":
        cfg.rope_neox, cfg.fused_qkv, cfg.fused_gate_up = True, True, True
    if fam == "glm4":
        cfg.fused_qkv, cfg.fused_gate_up, cfg.post_norms = True, True, True
        cfg.attn_bias, cfg.attn_out_bias = True, False
        cfg.rope_dim = cfg.rope_dim or cfg.head_dim // 2
    if fam == "glm4moe":
        cfg.rope_neox, cfg.attn_bias, cfg.attn_out_bias = True, True, False
        cfg.rope_dim = cfg.rope_dim or cfg.head_dim // 2
        cfg.moe_gating, cfg.shared_expert_gated = "sigmoid", False
        if md is not None:
            cfg.moe_dense_layers = int(g("leading_dense_block_count", cfg.moe_dense_layers))
            cfg.moe_scale = float(g("expert_weights_scale", cfg.moe_scale))
            cfg.moe_norm_topk = bool(g("expert_weights_norm", cfg.moe_norm_topk))
            n_sh = int(g("expert_shared_count", 1 if cfg.shared_expert_ffn else 0))
            cfg.shared_expert_ffn = n_sh * cfg.expert_ffn if n_sh else 0
            # next-token-prediction blocks follow the model's own layers
            cfg.mtp_layers = int(g("nextn_predict_layers", 0))
            cfg.n_layers -= cfg.mtp_layers
    if fam == "gpt-oss":
        cfg.rope_neox, cfg.attn_sinks, cfg.attn_bias, cfg.swa_every = True, True, True, 2
        cfg.swiglu_limit = cfg.swiglu_limit or 7.0
    if fam in ("qwen3next", "qwen35", "qwen35moe"):
        cfg.rope_neox, cfg.qk_norm, cfg.attn_output_gate = True, True, True
    if fam == "llama4":
        # iRoPE: every 4th layer has no rotary embedding; the RoPE layers
        # normalise q and k per head by their RMS with no weight (not in the
        # 128-expert Maverick); experts scored by a sigmoid, no selection bias,
        # no renormalisation, the weight applied to the expert's input, an
        # ungated shared expert; dense and routed layers interleaved.
        # Reference: src/inference/split/loader/mod.rs:1346 (routing),
        # :2392 (NoPE layers, q/k norm after RoPE).
        cfg.rope_neox, cfg.nope_every = False, 4
        cfg.qk_rms_plain = cfg.n_experts != 128
        if cfg.n_experts:
            cfg.moe_gating, cfg.moe_norm_topk, cfg.moe_scale = "sigmoid", False, 1.0
            cfg.moe_sel_bias, cfg.moe_weight_input, cfg.shared_expert_gated = False, True, False
            cfg.moe_every = int(g("interleave_moe_layer_step", cfg.moe_every or 1))
            if md is not None and not cfg.shared_expert_ffn:
                cfg.shared_expert_ffn = cfg.expert_ffn
    if fam == "granite" and md is not None:
        # Llama read with four multipliers (llama.cpp's granite keys; 0 or 1
        # means none for the embedding and residual ones); the attention
        # multiplier is the generic attention.scale.  Reference:
        # src/inference/model_arch.rs:77-81, split/gguf_meta.rs:594.
        emb = float(g("embedding_scale", 0.0) or 0.0)
        cfg.embed_scale = emb if emb not in (0.0, 1.0) else cfg.embed_scale
        res = float(g("residual_scale", 0.0) or 0.0)
        cfg.residual_scale = res if res not in (0.0, 1.0) else 0.0
        lg = float(g("logit_scale", 0.0) or 0.0)
        cfg.logit_scale = lg if lg not in (0.0, 1.0) else 0.0
    if fam in ("qwen35", "qwen35moe") and md is not None:
        # Qwen 3.5 files count only the trunk in block_count; the block after it
        # (blk.{block_count}) is the next-token-prediction head
        cfg.mtp_layers = int(g("nextn_predict_layers", cfg.mtp_layers))
    return cfg


def to_gguf_metadata(cfg: ModelConfig) -> dict:
    a = _ARCH_KEYS[cfg.arch]
    md = {
        "general.name": cfg.name,
        f"{a}.block_count": cfg.n_layers + (cfg.mtp_layers if cfg.arch == "glm4moe" else 0),
        f"{a}.embedding_length": cfg.hidden,
        f"{a}.feed_forward_length": cfg.ffn,
        f"{a}.attention.head_count": cfg.n_heads,
        f"{a}.attention.head_count_kv": cfg.n_kv_heads,
        f"{a}.attention.key_length": cfg.head_dim,
        f"{a}.attention.value_length": cfg.head_dim,
        f"{a}.attention.layer_norm_rms_epsilon": float(cfg.rms_eps),
        f"{a}.rope.freq_base": float(cfg.rope_theta),
        f"{a}.rope.dimension_count": cfg.rot_dim,
        f"{a}.vocab_size": cfg.vocab,
    }
    rs = cfg.rope_scaling or {}
    if rs.get("type") in ("linear", "yarn"):
        md[f"{a}.rope.scaling.type"] = rs["type"]
        md[f"{a}.rope.scaling.factor"] = float(rs["factor"])
        md[f"{a}.rope.scaling.original_context_length"] = int(
            rs.get("original_max_position_embeddings", 4096))
    if cfg.n_experts:
        md[f"{a}.expert_count"] = cfg.n_experts
        md[f"{a}.expert_used_count"] = cfg.n_experts_used
        md[f"{a}.expert_feed_forward_length"] = cfg.expert_ffn
        if cfg.shared_expert_ffn:
            md[f"{a}.expert_shared_feed_forward_length"] = cfg.shared_expert_ffn
        if cfg.moe_gating == "sigmoid":
            md[f"{a}.expert_gating_func"] = 2
            md[f"{a}.expert_weights_scale"] = float(cfg.moe_scale)
            md[f"{a}.expert_weights_norm"] = bool(cfg.moe_norm_topk)
            md[f"{a}.expert_shared_count"] = cfg.shared_expert_ffn // max(1, cfg.expert_ffn)
        if cfg.moe_dense_layers:
            md[f"{a}.leading_dense_block_count"] = cfg.moe_dense_layers
    if cfg.mtp_layers:
        md[f"{a}.nextn_predict_layers"] = cfg.mtp_layers
    if cfg.arch == "llama4" and cfg.moe_every > 1:
        md[f"{a}.interleave_moe_layer_step"] = cfg.moe_every
    if cfg.arch == "granite":
        for key, v in (("embedding_scale", cfg.embed_scale), ("residual_scale", cfg.residual_scale),
                       ("logit_scale", cfg.logit_scale)):
            md[f"{a}.{key}"] = float(v or 1.0)
    if cfg.attn_scale:
        md[f"{a}.attention.scale"] = float(cfg.attn_scale)
    if cfg.sliding_window:
        md[f"{a}.attention.sliding_window"] = cfg.sliding_window
    if cfg.attn_softcap:
        md[f"{a}.attn_logit_softcapping"] = float(cfg.attn_softcap)
    if cfg.final_softcap:
        md[f"{a}.final_logit_softcapping"] = float(cfg.final_softcap)
    if cfg.full_attn_interval:
        md[f"{a}.full_attention_interval"] = cfg.full_attn_interval
        md[f"{a}.ssm.conv_kernel"] = cfg.ssm_conv_kernel
        md[f"{a}.ssm.group_count"] = cfg.ssm_k_heads
        md[f"{a}.ssm.time_step_rank"] = cfg.ssm_v_heads
        md[f"{a}.ssm.state_size"] = cfg.ssm_head_dim
        md[f"{a}.ssm.inner_size"] = cfg.ssm_v_heads * cfg.ssm_head_dim
    # Engine-specific keys (prefixed) carry what GGUF has no standard key for.
    md["swarmllm.config"] = __import__("json").dumps(cfg.to_dict())
    return md


def from_gguf_metadata(md: dict) -> ModelConfig:
    import json
    if "swarmllm.config" in md:
        return ModelConfig(**json.loads(md["swarmllm.config"]))
    arch = md["general.architecture"]
    fam = arch if arch in _FAMILIES else _ARCH_ALIASES.get(arch)
    if fam is None:
        raise ValueError(f"unsupported architecture {arch}")
    a = arch

    def g(k, d=None):
        return md.get(f"{a}.{k}", d)

    n_heads = g("attention.head_count")
    hidden = g("embedding_length")
    cfg = ModelConfig(name=md.get("general.name", arch), arch=fam, n_layers=g("block_count"),
                      hidden=hidden, n_heads=n_heads,
                      n_kv_heads=g("attention.head_count_kv", n_heads),
                      head_dim=g("attention.key_length", hidden // n_heads),
                      ffn=g("feed_forward_length", 0), vocab=g("vocab_size", 0),
                      rope_theta=g("rope.freq_base", 10000.0),
                      rms_eps=g("attention.layer_norm_rms_epsilon", 1e-5),
                      rope_dim=g("rope.dimension_count", 0))
    if g("expert_count"):
        cfg.n_experts = g("expert_count")
        cfg.n_experts_used = g("expert_used_count")
        cfg.expert_ffn = g("expert_feed_forward_length", cfg.ffn)
        cfg.shared_expert_ffn = g("expert_shared_feed_forward_length", 0)
    if g("attention.sliding_window"):
        cfg.sliding_window = g("attention.sliding_window")
    if g("rope.scaling.type") in ("linear", "yarn", "longrope"):
        cfg.rope_scaling = {"type": g("rope.scaling.type"), "factor": g("rope.scaling.factor", 1.0),
                            "original_max_position_embeddings": g("rope.scaling.original_context_length", 4096)}
        if g("rope.scaling.attn_factor"):
            cfg.rope_scaling["attn_factor"] = g("rope.scaling.attn_factor")
    if g("attention.scale"):
        cfg.attn_scale = float(g("attention.scale"))
    if fam in ("qwen3next", "qwen35", "qwen35moe"):
        # llama.cpp's keys: group_count = key heads, time_step_rank = value
        # heads, state_size = key head width, inner_size = value heads x width
        cfg.full_attn_interval = g("full_attention_interval", 4)
        cfg.ssm_conv_kernel = g("ssm.conv_kernel", 4)
        cfg.ssm_k_heads = g("ssm.group_count", cfg.ssm_k_heads)
        cfg.ssm_v_heads = g("ssm.time_step_rank", cfg.ssm_v_heads)
        cfg.ssm_head_dim = g("ssm.state_size", cfg.ssm_head_dim)
        inner = g("ssm.inner_size")
        if inner and cfg.ssm_v_heads and inner != cfg.ssm_v_heads * cfg.ssm_head_dim:
            raise ValueError("DeltaNet value heads wider than key heads are not supported")
    if fam in ("gemma", "gemma2", "gemma3") and not g("vocab_size"):
        cfg.vocab = len(md.get("tokenizer.ggml.tokens", [])) or cfg.vocab
    return apply_family(cfg, md, prefix=a)
