"""File order <-> kernel order of the gated-DeltaNet tensors.

The DeltaNet kernels (csrc/kernels/deltanet*.cu) and the CPU oracle read the
value heads GROUPED by key head -- value head h reads key head h // r, with
r = n_v_heads / n_k_heads -- and the beta and decay-rate projections stacked
as one [2 n_v, hidden] tensor ``ssm_ba`` (all betas, then all alphas).  GGUF
files order them by family (llama.cpp's ``qwen3next.cpp`` / ``qwen35.cpp``,
as the reference reads them in src/inference/layers/qwen35.rs:116-230):

* ``qwen3next``: value heads grouped (the kernels' order); ``ssm_ba`` holds,
  per key head, its group's r betas and then their r alphas.
* ``qwen35`` / ``qwen35moe``: value heads TILED -- file head f reads key head
  f % n_k -- and separate ``ssm_beta`` / ``ssm_alpha`` tensors.  Kernel head
  g = kh * r + j is file head j * n_k + kh.

GLM-4.5 (``glm4moe``), gpt-oss and the Qwen 3.5 / Qwen3-Next hybrids name
the norm before the feed-forward ``post_attention_norm`` (llama.cpp reads it
as ``attn_post_norm`` on the FFN input); the engine calls it ``ffn_norm``
like every other family's, so it is renamed on the way in and out.

``to_kernel`` turns a file tensor into the kernels' order when a GGUF is read
(whole rows move, still quantized; ``ssm_out``'s value heads are columns,
moved as whole blocks where a block fits in a head, else the tensor is
dequantized to F16); ``file_specs`` / ``to_file`` do the opposite for the
random-init GGUF writer.
"""
from __future__ import annotations

import numpy as np

from ..gguf import quants as Q

HYBRID_FAMILIES = ("qwen3next", "qwen35", "qwen35moe")
TILED_FAMILIES = ("qwen35", "qwen35moe")
# engine name suffix -> file name suffix, per family
RENAMES = {a: {"ffn_norm.weight": "post_attention_norm.weight"}
           for a in ("glm4moe", "gpt-oss", "qwen3next", "qwen35", "qwen35moe")}
LAYOUT_FAMILIES = HYBRID_FAMILIES + tuple(RENAMES)


def file_name(arch: str, name: str) -> str:
    for a, b in RENAMES.get(arch, {}).items():
        if name.endswith("." + a):
            return name[: -len(a)] + b
    return name


def engine_name(arch: str, name: str) -> str:
    """The inverse of file_name."""
    for a, b in RENAMES.get(arch, {}).items():
        if name.endswith("." + b):
            return name[: -len(b)] + a
    return name


def file_head(arch: str, g: int, nk: int, nv: int) -> int:
    """The file's value head for kernel head g."""
    if arch not in TILED_FAMILIES:
        return g
    r = nv // nk
    return (g % r) * nk + g // r


def head_perm(arch: str, nk: int, nv: int) -> np.ndarray:
    """perm[g] = file head of kernel head g."""
    return np.array([file_head(arch, g, nk, nv) for g in range(nv)], dtype=np.int64)


def value_rows(arch: str, nk: int, nv: int, dv: int, offset: int = 0) -> np.ndarray:
    """File rows of the value part (dv rows per head, starting at `offset`),
    in kernel order."""
    p = head_perm(arch, nk, nv)
    return (offset + p[:, None] * dv + np.arange(dv)[None, :]).reshape(-1)


def qkv_rows(arch: str, nk: int, nv: int, dk: int, dv: int) -> np.ndarray:
    """File rows of ``attn_qkv`` (and conv channels) in kernel order: q and k
    as they are, the values reordered."""
    keys = 2 * nk * dk
    return np.concatenate([np.arange(keys), value_rows(arch, nk, nv, dv, keys)])


def ba_rows(nk: int, nv: int) -> np.ndarray:
    """qwen3next ``ssm_ba`` file rows in kernel order ([betas | alphas])."""
    r = nv // nk
    beta = [(g // r) * 2 * r + g % r for g in range(nv)]
    alpha = [(g // r) * 2 * r + r + g % r for g in range(nv)]
    return np.array(beta + alpha, dtype=np.int64)


def _take_rows(raw: np.ndarray, qt: int, shape, rows: np.ndarray) -> np.ndarray:
    n = shape[0]
    return np.ascontiguousarray(raw.reshape(n, -1)[rows]).reshape(-1)


def _col_blocks(raw: np.ndarray, qt: int, shape, perm: np.ndarray, width: int):
    """Columns of `shape` = [rows, nv * width] regrouped head by head (kernel
    head g takes file head perm[g]).  Returns (bytes, qtype): the blocks move
    as they are when `width` is a whole number of blocks, else the tensor is
    dequantized and returned as F16."""
    rows, cols = shape
    vals, nbytes = Q.BLOCK[qt]
    if width % vals == 0:
        per_head = width // vals * nbytes
        a = raw.reshape(rows, len(perm), per_head)[:, perm, :]
        return np.ascontiguousarray(a).reshape(-1), qt
    f = Q.dequantize(raw.reshape(-1), qt).reshape(rows, len(perm), width)[:, perm, :]
    return np.ascontiguousarray(f.reshape(rows, cols).astype(np.float16)).view(np.uint8).reshape(-1), Q.F16


def kernel_name(arch: str, name: str) -> list[str]:
    """The file tensors a kernel-order tensor is made of."""
    if arch in TILED_FAMILIES and name.endswith("ssm_ba.weight"):
        base = name[: -len("ssm_ba.weight")]
        return [base + "ssm_beta.weight", base + "ssm_alpha.weight"]
    return [file_name(arch, name)]


def to_kernel(cfg, name: str, fetch):
    """(bytes, qtype, shape) of tensor `name` in kernel order; `fetch(n)`
    returns a file tensor as (numpy uint8 bytes, qtype, shape)."""
    arch = cfg.arch
    parts = kernel_name(arch, name)
    if arch not in HYBRID_FAMILIES or ".ssm_" not in name and not name.endswith(
            ("attn_qkv.weight", "attn_gate.weight")):
        return fetch(file_name(arch, name))
    nk, nv, d = cfg.ssm_k_heads, cfg.ssm_v_heads, cfg.ssm_head_dim
    layer = int(name.split(".")[1])
    if not cfg.is_linear_attn(layer):
        return fetch(name)
    if name.endswith("ssm_ba.weight"):
        if arch in TILED_FAMILIES:
            (b, qb, sb), (a, qa, sa) = fetch(parts[0]), fetch(parts[1])
            p = head_perm(arch, nk, nv)
            if qb != qa:   # stack as F32
                b = Q.quantize(Q.dequantize(b, qb).reshape(sb), Q.F32).reshape(-1)
                a = Q.quantize(Q.dequantize(a, qa).reshape(sa), Q.F32).reshape(-1)
                qb = Q.F32
            return (np.concatenate([_take_rows(b, qb, sb, p), _take_rows(a, qb, sa, p)]), qb,
                    (2 * nv, sb[1]))
        raw, qt, shape = fetch(name)
        return _take_rows(raw, qt, shape, ba_rows(nk, nv)), qt, shape
    raw, qt, shape = fetch(name)
    if arch not in TILED_FAMILIES:
        return raw, qt, shape
    if name.endswith(("attn_qkv.weight", "ssm_conv1d.weight")):
        return _take_rows(raw, qt, shape, qkv_rows(arch, nk, nv, d, d)), qt, shape
    if name.endswith("attn_gate.weight"):
        return _take_rows(raw, qt, shape, value_rows(arch, nk, nv, d)), qt, shape
    if name.endswith(("ssm_dt.bias", "ssm_a")):
        return _take_rows(raw, qt, (shape[0], 1), head_perm(arch, nk, nv)), qt, shape
    if name.endswith("ssm_out.weight"):
        out, q2 = _col_blocks(raw, qt, shape, head_perm(arch, nk, nv), d)
        return out, q2, shape
    return raw, qt, shape


def file_specs(cfg, specs):
    """Kernel-order tensor specs -> the family's file tensors (name, shape, qtype)."""
    out = []
    for name, shape, qt in specs:
        if cfg.arch in TILED_FAMILIES and name.endswith("ssm_ba.weight"):
            half = (shape[0] // 2, shape[1])
            for n in kernel_name(cfg.arch, name):
                out.append((n, half, qt))
        else:
            out.append((file_name(cfg.arch, name), shape, qt))
    return out


def to_file(cfg, name: str, shape, qt: int, kernel_get):
    """Bytes of file tensor `name` from the kernel-order tensors
    (`kernel_get(n)` -> numpy uint8 bytes): the inverse of to_kernel, at the
    float level for column moves (the random-init writer's use)."""
    arch = cfg.arch
    name = engine_name(arch, name)
    if arch not in HYBRID_FAMILIES or ".ssm_" not in name and not name.endswith(
            ("attn_qkv.weight", "attn_gate.weight")):
        return kernel_get(name)
    layer = int(name.split(".")[1])
    if not cfg.is_linear_attn(layer):
        return kernel_get(name)
    nk, nv, d = cfg.ssm_k_heads, cfg.ssm_v_heads, cfg.ssm_head_dim

    def inv(perm):
        q = np.empty_like(perm)
        q[perm] = np.arange(len(perm))
        return q
    if arch not in TILED_FAMILIES:
        raw = kernel_get(name)
        if name.endswith("ssm_ba.weight"):
            return _take_rows(raw, qt, shape, inv(ba_rows(nk, nv)))
        return raw
    p = head_perm(arch, nk, nv)
    if name.endswith(("ssm_beta.weight", "ssm_alpha.weight")):
        base = name[: name.rindex("ssm_")]
        raw = kernel_get(base + "ssm_ba.weight")
        rows = raw.reshape(2 * nv, -1)
        half = rows[:nv] if name.endswith("ssm_beta.weight") else rows[nv:]
        return np.ascontiguousarray(half[inv(p)]).reshape(-1)
    raw = kernel_get(name)
    if name.endswith(("attn_qkv.weight", "ssm_conv1d.weight")):
        return _take_rows(raw, qt, shape, inv(qkv_rows(arch, nk, nv, d, d)))
    if name.endswith("attn_gate.weight"):
        return _take_rows(raw, qt, shape, inv(value_rows(arch, nk, nv, d)))
    if name.endswith(("ssm_dt.bias", "ssm_a")):
        return _take_rows(raw, qt, (shape[0], 1), inv(p))
    if name.endswith("ssm_out.weight"):
        out, q2 = _col_blocks(raw, qt, shape, inv(p), d)
        if q2 != qt:   # requantize the moved columns in the file's type
            f = Q.dequantize(out, q2).reshape(shape)
            out = Q.quantize(f, qt).reshape(-1)
        return out
    return raw
