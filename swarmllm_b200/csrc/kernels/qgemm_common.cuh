// Register-level weight dequantizers shared by the tensor-core GEMMs
// (qgemm_tc.cu: dense Q4_K, moe_tc.cu: grouped expert GEMMs).  Each turns one
// weight row's share of a 256-wide K unit into 16-bit pairs written straight
// into TMEM, where tcgen05.mma reads its A operand.
//
// TMEM A layout (kind::f16, A from tensor memory): lane = weight row, 32-bit
// column c holds K values (2c, 2c+1) with the even one in the low half.
#pragma once
#include "common.cuh"
#include "tc_utils.cuh"

namespace swarm {
using tc::tmem_st_x16;

SW_DEVICE __half2 u32_as_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }
SW_DEVICE uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// ----------------------------------------------------------------- Q4_K
constexpr int kQ4kRowBytes = 144;  // 128 B permuted nibbles + 16 B (d, dmin, scales)

// 8 permuted nibbles -> 4 fp16 pairs (K order), scale s, min mb.  The nibble
// order (0,2,4,6,1,3,5,7) lets one mask produce (1024 + q) pairs.
// (a & b) | c as one LOP3 (the compiler does not always fuse the pair)
SW_DEVICE uint32_t and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

SW_DEVICE void dq_word(uint32_t x, __half2 S, __half2 S16, __half2 MB, uint32_t* out) {
  const uint32_t MAGIC = 0x64006400u;
  const __half2 K1024 = u32_as_h2(0x64006400u);
  const uint32_t hi = x >> 8;
  __half2 c0 = __hsub2(u32_as_h2(and_or(x, 0x000F000Fu, MAGIC)), K1024);
  __half2 c1 = __hsub2(u32_as_h2(and_or(x, 0x00F000F0u, MAGIC)), K1024);
  __half2 c2 = __hsub2(u32_as_h2(and_or(hi, 0x000F000Fu, MAGIC)), K1024);
  __half2 c3 = __hsub2(u32_as_h2(and_or(hi, 0x00F000F0u, MAGIC)), K1024);
  out[0] = h2_as_u32(__hfma2(c0, S, MB));
  out[1] = h2_as_u32(__hfma2(c1, S16, MB));
  out[2] = h2_as_u32(__hfma2(c2, S, MB));
  out[3] = h2_as_u32(__hfma2(c3, S16, MB));
}

// (d*sc_j, dmin*m_j) for the 8 sub-blocks from the 16-byte header
// {f16 d, f16 dmin, u8 scales[12]}; constant byte indices keep it in registers.
SW_DEVICE void q4k_decode_scales(const uint4& hdr, float* s, float* mb) {
  const float d = half_bits_to_f((uint16_t)(hdr.x & 0xFFFF));
  const float dmin = half_bits_to_f((uint16_t)(hdr.x >> 16));
  const uint32_t w0 = hdr.y, w1 = hdr.z, w2 = hdr.w;
#define SB(i) ((int)((((i) < 4 ? w0 : ((i) < 8 ? w1 : w2)) >> (8 * ((i) & 3))) & 0xFF))
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    int sc, m;
    if (j < 4) {
      sc = SB(j) & 63;
      m = SB(j + 4) & 63;
    } else {
      sc = (SB(j + 4) & 0xF) | ((SB(j - 4) >> 6) << 4);
      m = (SB(j + 4) >> 4) | ((SB(j) >> 6) << 4);
    }
    s[j] = d * (float)sc;
    mb[j] = dmin * (float)m;
  }
#undef SB
}

// fp32 d * sc_j and dmin * m_j from the 16-byte header, with packed byte
// masks and the 2^23 float trick for the byte -> float conversions (exact).
SW_DEVICE void q4k_scales_f32(const uint4& hdr, float* s, float* mb) {
  const float d = half_bits_to_f((uint16_t)(hdr.x & 0xFFFF));
  const float dmin = half_bits_to_f((uint16_t)(hdr.x >> 16));
  const uint32_t w0 = hdr.y, w1 = hdr.z, w2 = hdr.w;
  const uint32_t sv[2] = {w0 & 0x3F3F3F3Fu, and_or(w0 >> 2, 0x30303030u, w2 & 0x0F0F0F0Fu)};
  const uint32_t mv[2] = {w1 & 0x3F3F3F3Fu, and_or(w1 >> 2, 0x30303030u, (w2 >> 4) & 0x0F0F0F0Fu)};
  const float M23 = 8388608.f;   // float bits 0x4B0000bb = 2^23 + bb
#pragma unroll
  for (int g = 0; g < 2; ++g)
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      s[4 * g + b] = d * (__int_as_float((int)__byte_perm(sv[g], 0x4B000000u, 0x7650u + b)) - M23);
      mb[4 * g + b] =
          dmin * (__int_as_float((int)__byte_perm(mv[g], 0x4B000000u, 0x7650u + b)) - M23);
    }
}

// The 8 sub-block scales and mins as fp16 pairs, with packed integer ops:
// S[i] = (d*sc_2i, d*sc_2i+1), NM[i] = (-dmin*m_2i, -dmin*m_2i+1).  Each 6-bit
// value is placed under the 0x64 exponent byte (1024 + v), 1024 is subtracted
// exactly and one HMUL2 applies d: the same single rounding as fp32 d*sc
// converted to fp16.
SW_DEVICE void q4k_scales_h2(const uint4& hdr, __half2 (&S)[4], __half2 (&NM)[4]) {
  const uint32_t w0 = hdr.y, w1 = hdr.z, w2 = hdr.w;
  const uint32_t sc03 = w0 & 0x3F3F3F3Fu, m03 = w1 & 0x3F3F3F3Fu;
  const uint32_t sc47 = and_or(w0 >> 2, 0x30303030u, w2 & 0x0F0F0F0Fu);
  const uint32_t m47 = and_or(w1 >> 2, 0x30303030u, (w2 >> 4) & 0x0F0F0F0Fu);
  const __half2 K1024 = u32_as_h2(0x64006400u);
  const __half2 d2 = u32_as_h2((hdr.x & 0xFFFFu) * 0x10001u);
  const __half2 nd2 = __hneg2(u32_as_h2((hdr.x >> 16) * 0x10001u));
  const uint32_t sv[2] = {sc03, sc47}, mv[2] = {m03, m47};
#pragma unroll
  for (int g = 0; g < 2; ++g) {
    S[2 * g] = __hmul2(__hsub2(u32_as_h2(__byte_perm(sv[g], 0x64646464u, 0x5140u)), K1024), d2);
    S[2 * g + 1] =
        __hmul2(__hsub2(u32_as_h2(__byte_perm(sv[g], 0x64646464u, 0x5342u)), K1024), d2);
    NM[2 * g] = __hmul2(__hsub2(u32_as_h2(__byte_perm(mv[g], 0x64646464u, 0x5140u)), K1024), nd2);
    NM[2 * g + 1] =
        __hmul2(__hsub2(u32_as_h2(__byte_perm(mv[g], 0x64646464u, 0x5342u)), K1024), nd2);
  }
}

// Sub-block c (K 32c .. 32c+31) of one row's superblock as the 16 32-bit
// TMEM columns [16c, 16c + 16) of the unit, in registers, from the fp16
// scale pairs of q4k_scales_h2.
SW_DEVICE void dq_chunk_h2(const uint4 (&q)[8], const __half2 (&S)[4], const __half2 (&NM)[4],
                           int c, uint32_t (&out)[16]) {
  const uint32_t* qw = reinterpret_cast<const uint32_t*>(q);
  const __half2 SIXTEENTH = u32_as_h2(0x2C002C00u);
  const __half2 Sp = S[c >> 1], Mp = NM[c >> 1];
  const __half2 Sj = (c & 1) ? __high2half2(Sp) : __low2half2(Sp);
  const __half2 MB = (c & 1) ? __high2half2(Mp) : __low2half2(Mp);
  const __half2 S16 = __hmul2(Sj, SIXTEENTH);
#pragma unroll
  for (int w4 = 0; w4 < 4; ++w4) dq_word(qw[4 * c + w4], Sj, S16, MB, out + 4 * w4);
}

// The 64 columns of half h from registers into TMEM (taddr: the unit's column 0).
SW_DEVICE void store_half(uint32_t taddr, int h, const uint32_t (&cols)[64]) {
#pragma unroll
  for (int k = 0; k < 4; ++k) tmem_st_x16(taddr + 64 * h + 16 * k, cols + 16 * k);
}

// Half h (chunks 4h .. 4h+3) of a format into registers.
template <class F>
SW_DEVICE void dq_half_regs(const typename F::Regs& r, int h, uint32_t (&out)[64]) {
#pragma unroll
  for (int k = 0; k < 4; ++k)
    F::dq_chunk(r, 4 * h + k, *reinterpret_cast<uint32_t(*)[16]>(out + 16 * k));
}

// A whole unit, chunk by chunk, straight into TMEM (16 registers live at a time).
template <class F>
SW_DEVICE void dq_unit_store(const typename F::Regs& r, uint32_t taddr) {
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    uint32_t cols[16];
    F::dq_chunk(r, c, cols);
    tmem_st_x16(taddr + 16 * c, cols);
  }
}

// Dequantize one row's superblock (256 K values) into the unit's 128 TMEM columns.
SW_DEVICE void dq_unit(const uint4 (&q)[8], const float* sc, const float* mb, uint32_t taddr) {
  const uint32_t* qw = reinterpret_cast<const uint32_t*>(q);
#pragma unroll
  for (int sub = 0; sub < 8; ++sub) {
    const __half2 S = __float2half2_rn(sc[sub]), S16 = __float2half2_rn(sc[sub] * 0.0625f);
    const __half2 MB = __float2half2_rn(-mb[sub]);
    uint32_t cols[16];
#pragma unroll
    for (int w4 = 0; w4 < 4; ++w4) dq_word(qw[4 * sub + w4], S, S16, MB, cols + 4 * w4);
    tmem_st_x16(taddr + sub * 16, cols);
  }
}

// ----------------------------------------------------------------- MXFP4
// Repacked MXFP4 (OCP MX: E2M1 values, one E8M0 scale per 32): a row's share
// of a 256-K unit is 8 scale bytes followed by 8 blocks x 16 B of nibbles
// (136 B; a trailing partial unit keeps the 8 scale bytes and only its blocks).
// Inside a block, 32-bit word w holds K = 8w..8w+7: nibble i (bits 4i..4i+3)
// is K = 8w+2i and nibble 4+i (bits 16+4i..) is K = 8w+2i+1, so every pair
// shares one shift.
constexpr int kMxRowBytes = 136;

// E2M1 nibble s|e1 e0 m placed as bf16 bits (mag << 6) | (s << 15) is the
// exact value times 2^-126 (e = 0 lands on the bf16 subnormals, which have the
// same spacing as E2M1's), so one bf16 multiply by 2^(E-1) applies the block
// scale 2^(E-127) exactly.  Scales above 2^1 (E > 128) are clamped.
SW_DEVICE uint32_t mx_scale_bf16x2(uint32_t e8m0) {
  const uint32_t e = e8m0 > 128u ? 128u : e8m0;
  const uint32_t b = (e + 126u) << 7;  // bf16 bits of 2^(e-1)
  return b | (b << 16);
}

SW_DEVICE uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// One block word (8 nibbles) -> 4 bf16 pairs.
SW_DEVICE void dq_mx_word(uint32_t x, uint32_t scale2, uint32_t* out) {
  const uint32_t MAG = 0x01C001C0u, SGN = 0x80008000u;
  out[0] = bf16x2_mul(((x << 6) & MAG) | ((x << 12) & SGN), scale2);
  out[1] = bf16x2_mul(((x << 2) & MAG) | ((x << 8) & SGN), scale2);
  out[2] = bf16x2_mul(((x >> 2) & MAG) | ((x << 4) & SGN), scale2);
  out[3] = bf16x2_mul(((x >> 6) & MAG) | (x & SGN), scale2);
}

}  // namespace swarm
