"""GGML block quantization formats in NumPy: quantize, dequantize, random-init.

These are the CPU reference implementations of the formats the CUDA kernels
read (``csrc/kernels/quant_blocks.cuh``).  Byte layouts follow the GGUF file
format so files interoperate with other GGUF tools:

=========  ======  =====  ===================================================
type       values  bytes  layout
=========  ======  =====  ===================================================
Q4_0       32      18     f16 d; u8 qs[16]            x = d * (q - 8)
Q8_0       32      34     f16 d; i8 qs[32]            x = d * q
Q4_K       256     144    f16 d, dmin; u8 scales[12]; u8 qs[128]
                          x = d*sc_j*q - dmin*m_j (6-bit sc, m per 32)
Q6_K       256     210    u8 ql[128]; u8 qh[64]; i8 scales[16]; f16 d
IQ4_NL     32      18     f16 d; u8 qs[16]            x = d * CODE[q]
IQ4_XS     256     136    f16 d; u16 scales_h; u8 scales_l[4]; u8 qs[128]
MXFP4      32      17     u8 e8m0; u8 qs[16]          x = 2^(e-128) * E2M1x2[q]
=========  ======  =====  ===================================================

The quantizers are simple min/max (or abs-max) fits, not llama.cpp's search
based ones: they are used to make random-init test models, where the exact
rounding choice does not matter but the format must be exact.  The reference
gets the same formats from candle's k_quants
(vendor/candle/candle-core/src/quantized/k_quants.rs) and checks MXFP4/IQ4
against llama.cpp C reference code (examples/mxfp4_reference.c,
examples/iq4_reference.c); here the dequantizers are checked against the
CUDA kernels instead.
"""
from __future__ import annotations

import numpy as np

# GGML type ids (GGUF spec).
F32, F16, Q4_0, Q8_0, Q4_K, Q6_K, IQ4_NL, IQ4_XS, BF16, MXFP4 = 0, 1, 2, 8, 12, 14, 20, 23, 30, 39

TYPE_NAMES = {F32: "F32", F16: "F16", Q4_0: "Q4_0", Q8_0: "Q8_0", Q4_K: "Q4_K", Q6_K: "Q6_K",
              IQ4_NL: "IQ4_NL", IQ4_XS: "IQ4_XS", BF16: "BF16", MXFP4: "MXFP4"}
NAME_TO_TYPE = {v: k for k, v in TYPE_NAMES.items()}

# (values per block, bytes per block)
BLOCK = {F32: (1, 4), F16: (1, 2), BF16: (1, 2), Q4_0: (32, 18), Q8_0: (32, 34),
         Q4_K: (256, 144), Q6_K: (256, 210), IQ4_NL: (32, 18), IQ4_XS: (256, 136),
         MXFP4: (32, 17)}

IQ4_CODE = np.array([-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113],
                    dtype=np.float32)
MXFP4_CODE = np.array([0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12], dtype=np.float32)


def nbytes(qtype: int, n_values: int) -> int:
    bv, bb = BLOCK[qtype]
    assert n_values % bv == 0, f"{n_values} not a multiple of block {bv}"
    return n_values // bv * bb


def _f16_bytes(a: np.ndarray) -> np.ndarray:
    return a.astype(np.float16).view(np.uint8).reshape(a.shape + (2,))


def _f16_from(b: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(b).view(np.float16)[..., 0].astype(np.float32)


def _nearest_code(x: np.ndarray, code: np.ndarray) -> np.ndarray:
    return np.abs(x[..., None] - code).argmin(-1).astype(np.uint8)


# --------------------------------------------------------------------------- quantize
def quantize(x: np.ndarray, qtype: int) -> np.ndarray:
    """Quantize float rows (last dim contiguous) -> uint8 [..., row_bytes]."""
    x = np.asarray(x, dtype=np.float32)
    lead, n = x.shape[:-1], x.shape[-1]
    if qtype == F32:
        return x.view(np.uint8).reshape(lead + (n * 4,)).copy()
    if qtype == F16:
        return x.astype(np.float16).view(np.uint8).reshape(lead + (n * 2,)).copy()
    if qtype == BF16:
        u = x.view(np.uint32)
        r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
        return r.view(np.uint8).reshape(lead + (n * 2,)).copy()
    bv, bb = BLOCK[qtype]
    blocks = x.reshape(-1, bv)
    out = {Q4_0: _q4_0, Q8_0: _q8_0, Q4_K: _q4_k, Q6_K: _q6_k, IQ4_NL: _iq4_nl,
           IQ4_XS: _iq4_xs, MXFP4: _mxfp4}[qtype](blocks)
    assert out.shape[-1] == bb
    return out.reshape(lead + (n // bv * bb,))


def _q8_0(b):
    amax = np.abs(b).max(-1)
    d = (amax / 127.0).astype(np.float16).astype(np.float32)
    inv = np.where(d > 0, 1.0 / np.where(d > 0, d, 1), 0)
    q = np.clip(np.rint(b * inv[:, None]), -127, 127).astype(np.int8)
    return np.concatenate([_f16_bytes(d), q.view(np.uint8)], -1)


def _q4_0(b):
    idx = np.abs(b).argmax(-1)
    amax = b[np.arange(len(b)), idx]
    d = (amax / -8.0).astype(np.float16).astype(np.float32)
    inv = np.where(d != 0, 1.0 / np.where(d != 0, d, 1), 0)
    q = np.clip(np.rint(b * inv[:, None]) + 8, 0, 15).astype(np.uint8)
    qs = q[:, :16] | (q[:, 16:] << 4)
    return np.concatenate([_f16_bytes(d), qs], -1)


def _iq4_nl(b):
    amax = np.abs(b).max(-1)
    d = (amax / 127.0).astype(np.float16).astype(np.float32)
    inv = np.where(d > 0, 1.0 / np.where(d > 0, d, 1), 0)
    q = _nearest_code(b * inv[:, None], IQ4_CODE)
    qs = q[:, :16] | (q[:, 16:] << 4)
    return np.concatenate([_f16_bytes(d), qs], -1)


def _mxfp4(b):
    amax = np.abs(b).max(-1)
    # smallest e with 12 * 2^(e-128) >= amax
    with np.errstate(divide="ignore"):
        e = np.where(amax > 0, np.ceil(np.log2(np.maximum(amax, 1e-38) / 12.0)) + 128, 0)
    e = np.clip(e, 0, 254).astype(np.uint8)
    d = np.ldexp(1.0, e.astype(np.int32) - 128).astype(np.float32)
    q = _nearest_code(b / d[:, None], MXFP4_CODE)
    qs = q[:, :16] | (q[:, 16:] << 4)
    return np.concatenate([e[:, None], qs], -1)


def _pack_q4k_scales(sc, m):
    """sc, m: [nb, 8] ints 0..63 -> [nb, 12] bytes."""
    s = np.zeros((sc.shape[0], 12), np.uint8)
    for j in range(4):
        s[:, j] = (sc[:, j] & 63) | ((sc[:, j + 4] >> 4) << 6)
        s[:, j + 4] = (m[:, j] & 63) | ((m[:, j + 4] >> 4) << 6)
        s[:, j + 8] = (sc[:, j + 4] & 0xF) | ((m[:, j + 4] & 0xF) << 4)
    return s


def _unpack_q4k_scales(s):
    sc = np.zeros(s.shape[:-1] + (8,), np.int32)
    m = np.zeros_like(sc)
    s = s.astype(np.int32)
    for j in range(8):
        if j < 4:
            sc[..., j] = s[..., j] & 63
            m[..., j] = s[..., j + 4] & 63
        else:
            sc[..., j] = (s[..., j + 4] & 0xF) | ((s[..., j - 4] >> 6) << 4)
            m[..., j] = (s[..., j + 4] >> 4) | ((s[..., j] >> 6) << 4)
    return sc, m


def _q4_k(b):
    nb = b.shape[0]
    sub = b.reshape(nb, 8, 32)
    mn = np.minimum(sub.min(-1), 0.0)
    mx = sub.max(-1)
    scale = (mx - mn) / 15.0
    mins = -mn
    d = (scale.max(-1) / 63.0).astype(np.float16).astype(np.float32)
    dmin = (mins.max(-1) / 63.0).astype(np.float16).astype(np.float32)
    sc = np.clip(np.rint(scale / np.where(d > 0, d, 1)[:, None]), 0, 63).astype(np.int32)
    m = np.clip(np.rint(mins / np.where(dmin > 0, dmin, 1)[:, None]), 0, 63).astype(np.int32)
    ds = d[:, None] * sc
    dm = dmin[:, None] * m
    q = np.rint((sub + dm[..., None]) / np.where(ds > 0, ds, 1)[..., None])
    q = np.clip(np.where(ds[..., None] > 0, q, 0), 0, 15).astype(np.uint8).reshape(nb, 256)
    qs = np.zeros((nb, 128), np.uint8)
    for g in range(4):
        qs[:, 32 * g:32 * g + 32] = q[:, 64 * g:64 * g + 32] | (q[:, 64 * g + 32:64 * g + 64] << 4)
    return np.concatenate([_f16_bytes(d), _f16_bytes(dmin), _pack_q4k_scales(sc, m), qs], -1)


def _q6_k(b):
    nb = b.shape[0]
    sub = b.reshape(nb, 16, 16)
    amax = np.abs(sub).max(-1)
    scale = amax / 32.0
    d = (np.abs(scale).max(-1) / 127.0).astype(np.float16).astype(np.float32)
    sc = np.clip(np.rint(scale / np.where(d > 0, d, 1)[:, None]), -128, 127).astype(np.int8)
    ds = d[:, None] * sc.astype(np.float32)
    q = np.rint(sub / np.where(ds != 0, ds, 1)[..., None])
    q = (np.clip(np.where(ds[..., None] != 0, q, 0), -32, 31) + 32).astype(np.uint8).reshape(nb, 256)
    ql = np.zeros((nb, 128), np.uint8)
    qh = np.zeros((nb, 64), np.uint8)
    for n in range(2):
        base = 128 * n
        q0, q1 = q[:, base:base + 32], q[:, base + 32:base + 64]
        q2, q3 = q[:, base + 64:base + 96], q[:, base + 96:base + 128]
        ql[:, 64 * n:64 * n + 32] = (q0 & 0xF) | ((q2 & 0xF) << 4)
        ql[:, 64 * n + 32:64 * n + 64] = (q1 & 0xF) | ((q3 & 0xF) << 4)
        qh[:, 32 * n:32 * n + 32] = (q0 >> 4) | ((q1 >> 4) << 2) | ((q2 >> 4) << 4) | ((q3 >> 4) << 6)
    return np.concatenate([ql, qh, sc.view(np.uint8), _f16_bytes(d)], -1)


def _iq4_xs(b):
    nb = b.shape[0]
    sub = b.reshape(nb, 8, 32)
    s = np.abs(sub).max(-1) / 127.0
    d = (s.max(-1) / 31.0).astype(np.float16).astype(np.float32)
    ls = np.clip(np.rint(s / np.where(d > 0, d, 1)[:, None]) + 32, 0, 63).astype(np.int32)
    dl = d[:, None] * (ls - 32)
    q = _nearest_code(sub / np.where(dl != 0, dl, 1)[..., None], IQ4_CODE).reshape(nb, 8, 32)
    qs = (q[..., :16] | (q[..., 16:] << 4)).reshape(nb, 128)
    sh = np.zeros(nb, np.uint16)
    sl = np.zeros((nb, 4), np.uint8)
    for ib in range(8):
        sh |= ((ls[:, ib] >> 4) & 3).astype(np.uint16) << (2 * ib)
        sl[:, ib // 2] |= ((ls[:, ib] & 0xF) << (4 * (ib % 2))).astype(np.uint8)
    return np.concatenate([_f16_bytes(d), sh.view(np.uint8).reshape(nb, 2), sl, qs], -1)


# --------------------------------------------------------------------------- dequantize
def dequantize(data: np.ndarray, qtype: int, n_values: int | None = None) -> np.ndarray:
    """uint8 [..., row_bytes] -> float32 [..., n]."""
    data = np.ascontiguousarray(data, dtype=np.uint8)
    lead = data.shape[:-1]
    if qtype == F32:
        return data.view(np.float32).reshape(lead + (-1,)).copy()
    if qtype == F16:
        return data.view(np.float16).astype(np.float32).reshape(lead + (-1,))
    if qtype == BF16:
        return (data.view(np.uint16).astype(np.uint32) << 16).view(np.float32).reshape(lead + (-1,))
    bv, bb = BLOCK[qtype]
    blocks = data.reshape(-1, bb)
    out = {Q4_0: _dq4_0, Q8_0: _dq8_0, Q4_K: _dq4_k, Q6_K: _dq6_k, IQ4_NL: _diq4_nl,
           IQ4_XS: _diq4_xs, MXFP4: _dmxfp4}[qtype](blocks)
    return out.astype(np.float32, copy=False).reshape(lead + (-1,))


def _dq8_0(b):
    return _f16_from(b[:, 0:2])[:, None] * b[:, 2:].view(np.int8).astype(np.float32)


def _nib(qs):
    return np.concatenate([qs & 0xF, qs >> 4], -1)


def _dq4_0(b):
    return _f16_from(b[:, 0:2])[:, None] * (_nib(b[:, 2:18]).astype(np.float32) - 8)


def _diq4_nl(b):
    return _f16_from(b[:, 0:2])[:, None] * IQ4_CODE[_nib(b[:, 2:18])]


def _dmxfp4(b):
    d = np.ldexp(1.0, b[:, 0].astype(np.int32) - 128).astype(np.float32)
    return d[:, None] * MXFP4_CODE[_nib(b[:, 1:17])]


def _dq4_k(b):
    nb = b.shape[0]
    d = _f16_from(b[:, 0:2])
    dmin = _f16_from(b[:, 2:4])
    sc, m = _unpack_q4k_scales(b[:, 4:16])
    qs = b[:, 16:144]
    q = np.zeros((nb, 256), np.float32)
    for g in range(4):
        q[:, 64 * g:64 * g + 32] = qs[:, 32 * g:32 * g + 32] & 0xF
        q[:, 64 * g + 32:64 * g + 64] = qs[:, 32 * g:32 * g + 32] >> 4
    q = q.reshape(nb, 8, 32)
    y = (d[:, None] * sc)[..., None] * q - (dmin[:, None] * m)[..., None]
    return y.reshape(nb, 256)


def _dq6_k(b):
    nb = b.shape[0]
    ql, qh = b[:, 0:128].astype(np.int32), b[:, 128:192].astype(np.int32)
    sc = b[:, 192:208].view(np.int8).astype(np.float32)
    d = _f16_from(b[:, 208:210])
    q = np.zeros((nb, 256), np.int32)
    for n in range(2):
        l0, l1 = ql[:, 64 * n:64 * n + 32], ql[:, 64 * n + 32:64 * n + 64]
        h = qh[:, 32 * n:32 * n + 32]
        q[:, 128 * n:128 * n + 32] = (l0 & 0xF) | ((h & 3) << 4)
        q[:, 128 * n + 32:128 * n + 64] = (l1 & 0xF) | (((h >> 2) & 3) << 4)
        q[:, 128 * n + 64:128 * n + 96] = (l0 >> 4) | (((h >> 4) & 3) << 4)
        q[:, 128 * n + 96:128 * n + 128] = (l1 >> 4) | (((h >> 6) & 3) << 4)
    q = (q - 32).reshape(nb, 16, 16).astype(np.float32)
    return ((d[:, None] * sc)[..., None] * q).reshape(nb, 256)


def _diq4_xs(b):
    nb = b.shape[0]
    d = _f16_from(b[:, 0:2])
    sh = b[:, 2:4].copy().view(np.uint16)[:, 0].astype(np.int32)
    sl = b[:, 4:8].astype(np.int32)
    qs = b[:, 8:136].reshape(nb, 8, 16)
    out = np.zeros((nb, 8, 32), np.float32)
    for ib in range(8):
        ls = ((sl[:, ib // 2] >> (4 * (ib % 2))) & 0xF) | (((sh >> (2 * ib)) & 3) << 4)
        dl = d * (ls - 32)
        out[:, ib] = dl[:, None] * IQ4_CODE[_nib(qs[:, ib])]
    return out.reshape(nb, 256)


# --------------------------------------------------------------------------- random init
def random_quantized(rows: int, cols: int, qtype: int, std: float = 0.02,
                     rng: np.random.Generator | None = None) -> np.ndarray:
    """N(0, std) weights [rows, cols], quantized -> uint8 [rows, row_bytes]."""
    rng = rng or np.random.default_rng(0)
    w = rng.standard_normal((rows, cols), dtype=np.float32) * std
    return quantize(w, qtype)


def q4k_repack_host(blocks: np.ndarray, rows: int, K: int) -> np.ndarray:
    """Host mirror of the device repack (launch_q4k_repack): GGUF Q4_K
    [rows, K/256*144] -> [rows_pad/128, K/256, 128, 144] with nibble-permuted
    codes first and the 16-byte (d, dmin, scales) header last."""
    ksb = K // 256
    rows_pad = (rows + 127) // 128 * 128
    src = np.zeros((rows_pad, ksb, 144), np.uint8)
    src[:rows] = blocks.reshape(rows, ksb, 144)
    qs = src[..., 16:144]
    vals = np.zeros((rows_pad, ksb, 256), np.uint32)
    for g in range(4):
        vals[..., 64 * g:64 * g + 32] = qs[..., 32 * g:32 * g + 32] & 0xF
        vals[..., 64 * g + 32:64 * g + 64] = qs[..., 32 * g:32 * g + 32] >> 4
    perm = [0, 2, 4, 6, 1, 3, 5, 7]
    v = vals.reshape(rows_pad, ksb, 32, 8)
    words = np.zeros((rows_pad, ksb, 32), np.uint32)
    for p in range(8):
        words |= v[..., perm[p]] << (4 * p)
    out = np.zeros((rows_pad, ksb, 144), np.uint8)
    out[..., :128] = words.view(np.uint8).reshape(rows_pad, ksb, 128)
    out[..., 128:] = src[..., :16]
    return out.reshape(rows_pad // 128, 128, ksb, 144).transpose(0, 2, 1, 3).copy()


def _q6k_codes(b: np.ndarray) -> np.ndarray:
    """6-bit codes [..., 256] (unsigned, q + 32) of Q6_K blocks [..., 210]."""
    ql, qh = b[..., 0:128].astype(np.uint32), b[..., 128:192].astype(np.uint32)
    q = np.zeros(b.shape[:-1] + (256,), np.uint32)
    for n in range(2):
        l0, l1 = ql[..., 64 * n:64 * n + 32], ql[..., 64 * n + 32:64 * n + 64]
        h = qh[..., 32 * n:32 * n + 32]
        q[..., 128 * n:128 * n + 32] = (l0 & 0xF) | ((h & 3) << 4)
        q[..., 128 * n + 32:128 * n + 64] = (l1 & 0xF) | (((h >> 2) & 3) << 4)
        q[..., 128 * n + 64:128 * n + 96] = (l0 >> 4) | (((h >> 4) & 3) << 4)
        q[..., 128 * n + 96:128 * n + 128] = (l1 >> 4) | (((h >> 6) & 3) << 4)
    return q


def _tile(out: np.ndarray, rows_pad: int, ksb: int, rb: int) -> np.ndarray:
    return out.reshape(rows_pad // 128, 128, ksb, rb).transpose(0, 2, 1, 3).copy()


def q6k_repack_host(blocks: np.ndarray, rows: int, K: int) -> np.ndarray:
    """Host mirror of the device Q6_K repack (launch_qfmt_repack, format 1):
    [rows_pad/128, K/256, 128, 224] = 32 low-nibble words (nibble order
    0,2,4,6,1,3,5,7 per 8 values), 16 crumb words (sub-block s: the top bits
    of K 16s+8e+2j at bit 8e+2j, of K+1 at bit 16+8e+2j) and 16 fp16 scales
    d * sc."""
    ksb = K // 256
    rows_pad = (rows + 127) // 128 * 128
    src = np.zeros((rows_pad, ksb, 210), np.uint8)
    src[:rows] = blocks.reshape(rows, ksb, 210)
    q = _q6k_codes(src)
    perm = [0, 2, 4, 6, 1, 3, 5, 7]
    v = (q & 0xF).reshape(rows_pad, ksb, 32, 8)
    lo = np.zeros((rows_pad, ksb, 32), np.uint32)
    for p in range(8):
        lo |= v[..., perm[p]] << (4 * p)
    hi = (q >> 4).reshape(rows_pad, ksb, 16, 2, 4, 2)      # s, e, j, (even, odd)
    cr = np.zeros((rows_pad, ksb, 16), np.uint32)
    for e in range(2):
        for j in range(4):
            cr |= hi[..., e, j, 0] << (8 * e + 2 * j)
            cr |= hi[..., e, j, 1] << (16 + 8 * e + 2 * j)
    d = _f16_from(src[..., 208:210])
    sc = src[..., 192:208].view(np.int8).astype(np.float32)
    scales = np.clip(d[..., None] * sc, -65504, 65504).astype(np.float16)
    out = np.zeros((rows_pad, ksb, 224), np.uint8)
    out[..., 0:128] = lo.view(np.uint8).reshape(rows_pad, ksb, 128)
    out[..., 128:192] = cr.view(np.uint8).reshape(rows_pad, ksb, 64)
    out[..., 192:224] = scales.view(np.uint8).reshape(rows_pad, ksb, 32)
    return _tile(out, rows_pad, ksb, 224)


def q80_repack_host(blocks: np.ndarray, rows: int, K: int) -> np.ndarray:
    """Host mirror of the device Q8_0 repack (format 2): [rows_pad/128, K/256,
    128, 272] = 256 codes q ^ 0x80 in K order, then 8 fp16 block scales."""
    ksb = K // 256
    rows_pad = (rows + 127) // 128 * 128
    src = np.zeros((rows_pad, ksb, 8, 34), np.uint8)
    src[:rows] = blocks.reshape(rows, ksb, 8, 34)
    out = np.zeros((rows_pad, ksb, 272), np.uint8)
    out[..., :256] = (src[..., 2:] ^ 0x80).reshape(rows_pad, ksb, 256)
    out[..., 256:] = src[..., :2].reshape(rows_pad, ksb, 16)
    out[rows:] = 0                                         # padding rows stay zero
    return _tile(out, rows_pad, ksb, 272)


def repacked_dequant_host(packed: np.ndarray, fmt: int, rows: int, K: int) -> np.ndarray:
    """fp32 [rows, K] from a repacked tensor (format 1 = Q6_K, 2 = Q8_0),
    decoded from the layout description alone, with the scale rounded to fp16
    as the kernels do: the oracle of the repacked-format kernels."""
    ksb = K // 256
    rb = {1: 224, 2: 272}[fmt]
    rows_pad = (rows + 127) // 128 * 128
    t = packed.reshape(rows_pad // 128, ksb, 128, rb).transpose(0, 2, 1, 3).reshape(rows_pad, ksb, rb)
    if fmt == 2:
        q = (t[..., :256] ^ 0x80).view(np.int8).astype(np.float32).reshape(rows_pad, ksb, 8, 32)
        d = t[..., 256:272].copy().view(np.float16).astype(np.float32)
        w = q * d[..., None]
    else:
        lo = t[..., :128].copy().view(np.uint32)           # [.., 32]
        cr = t[..., 128:192].copy().view(np.uint32)        # [.., 16]
        sc = t[..., 192:224].copy().view(np.float16).astype(np.float32)
        q = np.zeros((rows_pad, ksb, 256), np.int64)
        perm = [0, 2, 4, 6, 1, 3, 5, 7]
        for wi in range(32):
            for p in range(8):
                k = 8 * wi + perm[p]
                s, e, j, odd = k // 16, (k % 16) // 8, (k % 8) // 2, k % 2
                nib = (lo[..., wi] >> (4 * p)) & 0xF
                top = (cr[..., s] >> (16 * odd + 8 * e + 2 * j)) & 3
                q[..., k] = (nib | (top << 4)).astype(np.int64) - 32
        w = q.reshape(rows_pad, ksb, 16, 16).astype(np.float32) * sc[..., None]
    return w.reshape(rows_pad, K)[:rows]
