"""Repacked weight formats of the quantized tensor-core GEMM / GEMV (CPU).

The device kernels (csrc/kernels/qfmt.cuh) decode the repacked rows with
bit tricks: code bits OR-ed into the mantissa of fp16 1024.0, an exact
subtraction, one scale multiply.  These tests run the same word-level
operations with numpy (uint32 words reinterpreted as fp16 pairs) on the host
repack and compare with the GGUF dequantizer, so the layout and the masks and
shifts are checked without a GPU."""
import numpy as np
import pytest

from swarmllm_b200.gguf import quants as Q


def _h2(u):
    """uint32 words -> fp16 pairs [..., 2] (low half first)."""
    a = np.atleast_1d(np.asarray(u, np.uint32))
    return a.view(np.float16).reshape(np.shape(u) + (2,)).astype(np.float32)


def _and_or(a, m, c):
    return (np.uint32(a) & np.uint32(m)) | np.uint32(c)


def _q6k_word(x, h):
    """Mirror of q6k_word: pairs (q - 32) from a low-nibble word and its crumbs."""
    M = 0x64006400
    hi = np.uint32(x) >> np.uint32(8)
    h = np.uint32(h)
    c0 = _h2(_and_or(h << np.uint32(4), 0x00300030, _and_or(x, 0x000F000F, M))) - 1056
    c1 = _h2(_and_or(h << np.uint32(6), 0x03000300, _and_or(x, 0x00F000F0, M))) / 16 - 96
    c2 = _h2(_and_or(h, 0x00300030, _and_or(hi, 0x000F000F, M))) - 1056
    c3 = _h2(_and_or(h << np.uint32(2), 0x03000300, _and_or(hi, 0x00F000F0, M))) / 16 - 96
    return np.concatenate([c0, c1, c2, c3])      # K order k0..k7


def test_q6k_word_decode_matches_gguf():
    rng = np.random.default_rng(0)
    rows, K = 128, 512
    b = Q.quantize(rng.standard_normal((rows, K), dtype=np.float32) * 0.03, Q.Q6_K)
    codes = Q._q6k_codes(b.reshape(rows, K // 256, 210)).reshape(rows, K).astype(np.int64) - 32
    pk = Q.q6k_repack_host(b, rows, K)                     # [1, ksb, 128, 224]
    for sb in range(K // 256):
        for r in (0, 5, 77, 127):
            row = pk[0, sb, r]
            lo = row[:128].copy().view(np.uint32)
            cr = row[128:192].copy().view(np.uint32)
            got = []
            for s in range(16):
                for e in range(2):
                    h = cr[s] >> np.uint32(8) if e else cr[s]
                    got.append(_q6k_word(lo[2 * s + e], h))
            got = np.concatenate(got)
            assert np.array_equal(got, codes[r, 256 * sb:256 * sb + 256]), (sb, r)


def test_q80_word_decode_matches_gguf():
    rng = np.random.default_rng(1)
    rows, K = 128, 256
    b = Q.quantize(rng.standard_normal((rows, K), dtype=np.float32), Q.Q8_0)
    q = b.reshape(rows, 8, 34)[..., 2:].view(np.int8).reshape(rows, K).astype(np.int64)
    pk = Q.q80_repack_host(b, rows, K)
    for r in (0, 63, 127):
        words = pk[0, 0, r, :256].copy().view(np.uint32)
        got = []
        for x in words:
            # byte_perm(x, 0x64646464, 0x5140 / 0x5342): byte under the 0x64 exponent byte
            b0, b1, b2, b3 = [(int(x) >> (8 * i)) & 0xFF for i in range(4)]
            p0 = b0 | (0x64 << 8) | (b1 << 16) | (0x64 << 24)
            p1 = b2 | (0x64 << 8) | (b3 << 16) | (0x64 << 24)
            got.append(_h2(np.uint32(p0)) - 1152)
            got.append(_h2(np.uint32(p1)) - 1152)
        assert np.array_equal(np.concatenate(got), q[r])


@pytest.mark.parametrize("qt,fmt", [(Q.Q6_K, 1), (Q.Q8_0, 2)])
def test_repacked_layout_dequantizes(qt, fmt):
    """The repacked layout holds the same weights (Q6_K: scales rounded to fp16)."""
    rng = np.random.default_rng(2)
    rows, K = 200, 768                                    # padded to 256 rows
    w = rng.standard_normal((rows, K), dtype=np.float32) * 0.02
    b = Q.quantize(w, qt)
    ref = Q.dequantize(b, qt).reshape(rows, K)
    pk = (Q.q6k_repack_host if fmt == 1 else Q.q80_repack_host)(b, rows, K)
    assert pk.shape == (2, K // 256, 128, {1: 224, 2: 272}[fmt])
    got = Q.repacked_dequant_host(pk.reshape(-1), fmt, rows, K)
    rel = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert rel < (1e-3 if fmt == 1 else 1e-7), rel
    assert not pk[1, :, rows - 128:].any()                # padding rows are zero


def test_q6k_int8_bytes_match_codes():
    """Mirror of FmtQ6K::gemv_i8's byte rebuild: low nibbles with their crumbs
    shifted into each byte lane, in the int8 activations' order (K' = 0,4,1,5
    and 2,6,3,7), minus 32."""
    rng = np.random.default_rng(5)
    rows, K = 128, 256
    b = Q.quantize(rng.standard_normal((rows, K), dtype=np.float32) * 0.03, Q.Q6_K)
    codes = Q._q6k_codes(b.reshape(rows, 1, 210)).reshape(rows, K).astype(np.int64) - 32
    pk = Q.q6k_repack_host(b, rows, K)
    for r in (0, 5, 127):
        row = pk[0, 0, r]
        lo = row[:128].copy().view(np.uint32)
        cr = row[128:192].copy().view(np.uint32)
        for s in range(16):
            for e in range(2):
                x, h = int(lo[2 * s + e]), (int(cr[s]) >> 8 if e else int(cr[s]))
                L = ((h << 8) & 0x30003000) | ((h << 4) & 0x00300030) | (x & 0x0F0F0F0F)
                H = ((h << 6) & 0x30003000) | ((h << 2) & 0x00300030) | ((x >> 4) & 0x0F0F0F0F)
                got_lo = [((L >> (8 * i)) & 0xFF) - 32 for i in range(4)]
                got_hi = [((H >> (8 * i)) & 0xFF) - 32 for i in range(4)]
                base = 16 * s + 8 * e
                assert got_lo == [codes[r, base + k] for k in (0, 4, 1, 5)]
                assert got_hi == [codes[r, base + k] for k in (2, 6, 3, 7)]
