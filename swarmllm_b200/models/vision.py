"""Vision-language input: an image encoder read from an mmproj GGUF, and the
image rows it produces for the language model's prompt.

The encoder is a ViT: patch embedding (a strided convolution), optional class
token, learned position embeddings, optional pre-norm, pre-norm transformer
blocks (LayerNorm, multi-head attention with biases, LayerNorm, GELU MLP),
optional post-norm, then a projector into the language model's hidden size:

  mlp     LLaVA: patch features (class token dropped) -> linear -> GELU -> linear
  gemma3  Gemma 3: SigLIP features averaged over s x s patch squares ->
          RMSNorm -> linear (`mm.soft_emb_norm`, `mm.input_projection`)

Tensor names and metadata keys are those of llama.cpp's mmproj files
(`v.patch_embd`, `v.class_embd`, `v.position_embd`, `v.pre_ln`,
`v.blk.N.{ln1,attn_q,attn_k,attn_v,attn_out,ln2,ffn_up,ffn_down}`, `v.post_ln`,
`mm.0` / `mm.2`; `clip.vision.*`, `clip.projector_type`).  Legacy CLIP
conversions store the MLP expansion as `ffn_down`; that is detected from the
shapes.  A LLaVA file without `clip.vision.feature_layer` runs all its blocks
(the converter already dropped the last one); with one, that many.

The encoder runs once per image in plain PyTorch (it is not on the decode
path); the engine splices its rows into the prompt at the image marker
(engine.add_request(images=...)).

Reference behaviour: src/inference/vision.rs (preprocess_image:93,
VisionEncoder:488, LLaVA projector:564, Gemma 3 projection:605,
load_from_mmproj_gguf, encoder_depth:1560, image_spans:881).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch
import torch.nn.functional as F

# Marks an image's place in a token-id prompt (one per image, LLaVA's convention)
IMAGE_TOKEN = -200
MEDIA_MARKER = "<__media__>"   # the same mark in rendered chat text

CLIP_MEAN = (0.48145466, 0.4578275, 0.40821073)
CLIP_STD = (0.26862954, 0.26130258, 0.27577711)


@dataclass
class VisionConfig:
    image_size: int
    patch_size: int
    hidden: int
    heads: int
    blocks: int
    eps: float = 1e-6
    projector: str = "mlp"
    mean: tuple = CLIP_MEAN
    std: tuple = CLIP_STD
    gelu_tanh: bool = False
    pool: int = 4          # gemma3: side of the averaged square of patches

    @property
    def patches_per_side(self) -> int:
        return self.image_size // self.patch_size


class VisionEncoder:
    def __init__(self, cfg: VisionConfig, tensors: dict, llm_hidden: int, device="cpu",
                 dtype=torch.float32, depth: int | None = None):
        self.cfg, self.device, self.dtype = cfg, torch.device(device), dtype
        t = {k: torch.as_tensor(np.asarray(v, dtype=np.float32)).to(self.device, dtype)
             for k, v in tensors.items()}
        self.t = t
        self.depth = cfg.blocks if depth is None else depth
        self.llm_hidden = llm_hidden
        # legacy CLIP conversions name the expansion "ffn_down"
        fd = t.get("v.blk.0.ffn_down.weight")
        self.ffn_swapped = fd is not None and fd.shape[1] == cfg.hidden and fd.shape[0] != cfg.hidden

    # ------------------------------------------------------------------ loading
    @classmethod
    def from_gguf(cls, path: str, llm_hidden: int, device="cpu", dtype=torch.float32):
        from ..gguf.file import GGUFReader
        r = GGUFReader(path)
        md = r.metadata
        g = lambda k, d=None: md.get(k, d)
        ptype = str(g("clip.projector_type", "mlp"))
        if ptype not in ("mlp", "gemma3"):
            raise ValueError(f"projector type {ptype!r} is not supported (mlp, gemma3)")
        cfg = VisionConfig(image_size=int(g("clip.vision.image_size")),
                           patch_size=int(g("clip.vision.patch_size")),
                           hidden=int(g("clip.vision.embedding_length")),
                           heads=int(g("clip.vision.attention.head_count")),
                           blocks=int(g("clip.vision.block_count")),
                           eps=float(g("clip.vision.attention.layer_norm_epsilon", 1e-6)),
                           projector=ptype,
                           mean=tuple(g("clip.vision.image_mean", CLIP_MEAN)),
                           std=tuple(g("clip.vision.image_std", CLIP_STD)),
                           gelu_tanh=ptype == "gemma3",
                           pool=int(g("clip.vision.projector.scale_factor", 4)))
        depth = None
        fl = g("clip.vision.feature_layer")
        if ptype == "mlp" and fl is not None:
            fl = list(fl) if isinstance(fl, (list, tuple)) else [fl]
            if len(fl) != 1 or not 0 <= int(fl[0]) <= cfg.blocks:
                raise ValueError(f"feature layers {fl} are not supported")
            depth = int(fl[0])
        tensors = {name: r.tensor_float(name) for name in r.tensors}
        return cls(cfg, tensors, llm_hidden, device, dtype, depth)

    # ------------------------------------------------------------------ images
    def preprocess(self, image) -> torch.Tensor:
        """An image (PIL image, HxWx3 uint8 array or bytes of PNG/JPEG) -> a
        normalised [3, S, S] tensor: padded to a square with the mean colour
        (LLaVA) or stretched (Gemma 3), resized bicubically, then (x - mean) / std."""
        if isinstance(image, (bytes, bytearray)):
            import io

            from PIL import Image
            image = Image.open(io.BytesIO(image))
        if hasattr(image, "convert"):
            image = np.asarray(image.convert("RGB"))
        a = torch.as_tensor(np.asarray(image, dtype=np.float32) / 255.0)
        if a.ndim != 3 or a.shape[2] != 3:
            raise ValueError("expected an RGB image")
        x = a.permute(2, 0, 1)  # [3, H, W]
        S = self.cfg.image_size
        mean = torch.tensor(self.cfg.mean).view(3, 1, 1)
        std = torch.tensor(self.cfg.std).view(3, 1, 1)
        if self.cfg.projector == "mlp":  # letterbox to a square of the mean colour
            h, w = x.shape[1:]
            side = max(h, w)
            sq = mean.expand(3, side, side).clone()
            top, left = (side - h) // 2, (side - w) // 2
            sq[:, top:top + h, left:left + w] = x
            x = sq
        x = F.interpolate(x[None], size=(S, S), mode="bicubic", align_corners=False)[0].clamp(0, 1)
        return ((x - mean) / std).to(self.device, self.dtype)

    # ------------------------------------------------------------------ encoder
    def _ln(self, x, name):
        w, b = self.t[name + ".weight"], self.t.get(name + ".bias")
        return F.layer_norm(x, (x.shape[-1],), w, b, self.cfg.eps)

    def _lin(self, x, name):
        return F.linear(x, self.t[name + ".weight"], self.t.get(name + ".bias"))

    def _gelu(self, x):
        return F.gelu(x, approximate="tanh" if self.cfg.gelu_tanh else "none")

    @property
    def rows_per_image(self) -> int:
        n = self.cfg.patches_per_side
        if self.cfg.projector == "gemma3":
            return (n // self.cfg.pool) ** 2
        return n * n

    @torch.no_grad()
    def encode(self, images) -> torch.Tensor:
        """[n_images * rows_per_image, llm_hidden] image rows (fp32)."""
        c = self.cfg
        x = torch.stack([self.preprocess(im) for im in images])            # [B, 3, S, S]
        pe = self.t["v.patch_embd.weight"]                                 # [hidden, 3, p, p]
        h = F.conv2d(x, pe, self.t.get("v.patch_embd.bias"), stride=c.patch_size)
        h = h.flatten(2).transpose(1, 2)                                   # [B, n_patch, hidden]
        cls = "v.class_embd" in self.t
        if cls:
            h = torch.cat([self.t["v.class_embd"].view(1, 1, -1).expand(h.shape[0], 1, -1), h], 1)
        h = h + self.t["v.position_embd.weight"][: h.shape[1]]
        if "v.pre_ln.weight" in self.t:
            h = self._ln(h, "v.pre_ln")
        nh, hd = c.heads, c.hidden // c.heads
        up, down = ("ffn_down", "ffn_up") if self.ffn_swapped else ("ffn_up", "ffn_down")
        for i in range(self.depth):
            p = f"v.blk.{i}."
            y = self._ln(h, p + "ln1")
            B, N, _ = y.shape
            q = self._lin(y, p + "attn_q").view(B, N, nh, hd).transpose(1, 2)
            k = self._lin(y, p + "attn_k").view(B, N, nh, hd).transpose(1, 2)
            v = self._lin(y, p + "attn_v").view(B, N, nh, hd).transpose(1, 2)
            a = F.scaled_dot_product_attention(q, k, v)                  # bidirectional
            h = h + self._lin(a.transpose(1, 2).reshape(B, N, c.hidden), p + "attn_out")
            y = self._ln(h, p + "ln2")
            h = h + self._lin(self._gelu(self._lin(y, p + up)), p + down)
        if "v.post_ln.weight" in self.t and self.depth == c.blocks:
            h = self._ln(h, "v.post_ln")
        if cls:
            h = h[:, 1:]
        if c.projector == "mlp":
            out = self._lin(F.gelu(self._lin(h, "mm.0")), "mm.2")
        else:  # gemma3: average s x s squares of patches, RMS norm, project
            n = c.patches_per_side
            g = h.view(h.shape[0], n, n, -1).permute(0, 3, 1, 2)
            g = F.avg_pool2d(g, c.pool).flatten(2).transpose(1, 2)
            w = self.t["mm.soft_emb_norm.weight"]
            g = g * torch.rsqrt(g.pow(2).mean(-1, keepdim=True) + c.eps) * w
            proj = self.t["mm.input_projection.weight"]
            out = g @ proj if proj.shape[0] == c.hidden else g @ proj.T
        if out.shape[-1] != self.llm_hidden:
            raise ValueError(f"projector gives {out.shape[-1]} features, the model wants {self.llm_hidden}")
        return out.reshape(-1, self.llm_hidden).float()


def image_placeholders(rows: torch.Tensor, n: int, vocab: int) -> list[int]:
    """Token ids for an image's n rows: derived from the rows' content, so the
    prefix cache (which hashes token ids) never confuses two images.  The
    embeddings of these positions are replaced by the image rows."""
    import hashlib
    hsh = int.from_bytes(hashlib.sha256(rows.detach().cpu().numpy().tobytes()).digest()[:8], "little")
    return [int((hsh + 1_000_003 * i) % vocab) for i in range(n)]


def write_random_mmproj(path: str, image_size: int = 28, patch: int = 14, hidden: int = 64,
                        heads: int = 4, blocks: int = 2, llm_hidden: int = 256,
                        projector: str = "mlp", seed: int = 0, legacy_ffn: bool = False):
    """A small random mmproj GGUF (tests and synthetic runs)."""
    from ..gguf import quants as Q
    from ..gguf.file import GGUFWriter
    rng = np.random.default_rng(seed)
    w = GGUFWriter("clip")
    w.add("clip.projector_type", projector)
    w.add("clip.vision.image_size", image_size)
    w.add("clip.vision.patch_size", patch)
    w.add("clip.vision.embedding_length", hidden)
    w.add("clip.vision.feed_forward_length", 4 * hidden)
    w.add("clip.vision.attention.head_count", heads)
    w.add("clip.vision.block_count", blocks)
    w.add("clip.vision.attention.layer_norm_epsilon", 1e-6)
    w.add("clip.vision.image_mean", list(CLIP_MEAN))
    w.add("clip.vision.image_std", list(CLIP_STD))
    if projector == "gemma3":
        w.add("clip.vision.projector.scale_factor", 2)

    def put(name, *shape, scale=None):
        s = scale if scale is not None else 1.0 / math.sqrt(shape[-1])
        a = (rng.standard_normal(shape) * s).astype(np.float32)
        w.add_tensor(name, a, Q.F32, shape)

    n = (image_size // patch) ** 2
    put("v.patch_embd.weight", hidden, 3, patch, patch, scale=0.05)
    if projector == "mlp":
        put("v.class_embd", hidden, scale=0.02)
        put("v.position_embd.weight", n + 1, hidden, scale=0.02)
        put("v.pre_ln.weight", hidden, scale=0.1)
        put("v.pre_ln.bias", hidden, scale=0.01)
    else:
        put("v.position_embd.weight", n, hidden, scale=0.02)
    for i in range(blocks):
        p = f"v.blk.{i}."
        for nm in ("ln1", "ln2"):
            put(p + nm + ".weight", hidden, scale=0.1)
            put(p + nm + ".bias", hidden, scale=0.01)
        for nm in ("attn_q", "attn_k", "attn_v", "attn_out"):
            put(p + nm + ".weight", hidden, hidden)
            put(p + nm + ".bias", hidden, scale=0.01)
        expand, contract = ("ffn_down", "ffn_up") if legacy_ffn else ("ffn_up", "ffn_down")
        put(p + expand + ".weight", 4 * hidden, hidden)
        put(p + expand + ".bias", 4 * hidden, scale=0.01)
        put(p + contract + ".weight", hidden, 4 * hidden)
        put(p + contract + ".bias", hidden, scale=0.01)
    if projector == "mlp":
        put("mm.0.weight", llm_hidden, hidden)
        put("mm.0.bias", llm_hidden, scale=0.01)
        put("mm.2.weight", llm_hidden, llm_hidden)
        put("mm.2.bias", llm_hidden, scale=0.01)
    else:
        put("v.post_ln.weight", hidden, scale=0.1)
        put("v.post_ln.bias", hidden, scale=0.01)
        put("mm.soft_emb_norm.weight", hidden, scale=0.1)
        put("mm.input_projection.weight", hidden, llm_hidden)
    w.write(path)
