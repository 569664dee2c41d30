// Weight formats of the quantized GEMMs (qgemm_tc.cu on the tensor cores,
// qgemv_q4k.cu on the CUDA cores at 1..2 tokens).
//
// Every format is repacked once at load time into the same tiling,
// [row_tile][256-K superblock][128 rows][ROW_BYTES], so a 128-row x 256-K
// unit is one contiguous bulk copy and the kernels' pipelines, stream-K split
// and partial-slot format do not depend on the format.  A format supplies:
//   Regs           one weight row's share of a unit, in registers
//   load / prep    shared memory -> registers; scale decode (before any wait)
//   dq_chunk(c)    K [32c, 32c+32) -> the 16 TMEM columns [16c, 16c+16) as
//                  fp16 pairs, in registers (A operand of tcgen05.mma, lane =
//                  row, 32-bit column c = K values 2c, 2c+1); the GEMM stores
//                  them into TMEM
//   gemv_prep,     acc[t] += sum_k W[row][k] * X[t][k] on the CUDA cores
//   gemv<T>
//
// GGUF block layouts (gguf/quants.py has the CPU (de)quantizers):
//   Q4_K  {f16 d, f16 dmin, u8 scales[12], u8 qs[128]}      256 values
//   Q6_K  {u8 ql[128], u8 qh[64], i8 scales[16], f16 d}     256 values
//   Q8_0  {f16 d, i8 qs[32]}                                 32 values
// Repacked rows (this file's own layouts):
//   Q4_K  128 B nibbles (word w = K 8w..8w+7 in nibble order 0,2,4,6,1,3,5,7)
//         + the 16 B header                                            144 B
//   Q6_K  128 B low nibbles (same order) + 64 B high 2-bit "crumbs" + 16 fp16
//         sub-block scales d*sc                                        224 B
//         crumb word s covers K 16s..16s+15: for x-word e (0, 1) and pair j,
//         the crumb of K 16s+8e+2j sits at bit 8e+2j, of K+1 at bit 16+8e+2j,
//         so each pair's crumbs reach their fp16 mantissa bits by one shift.
//   Q8_0  256 B codes q ^ 0x80 (unsigned, K order) + 8 fp16 block scales 272 B
//
// All formats build fp16 values exactly the same way: the code bits are OR-ed
// into the mantissa of 1024.0 (0x6400), which gives 1024 + q exactly, and a
// subtraction of an exact constant leaves the integer (q - zero point), which
// one multiply scales (one rounding, as a dequantized fp16 weight has).
#pragma once
#include "qgemm_common.cuh"

namespace swarm {

enum : int { kFmtQ4K = 0, kFmtQ6K = 1, kFmtQ8_0 = 2, kNumQFmts = 3 };

SW_DEVICE uint32_t byte_perm(uint32_t a, uint32_t b, uint32_t sel) {
  return __byte_perm(a, b, sel);
}

// ----------------------------------------------------------------- Q4_K
struct FmtQ4K {
  static constexpr int ID = kFmtQ4K;
  static constexpr int ROW_BYTES = kQ4kRowBytes;
  static constexpr bool HAS_I8 = true, X8_NATURAL = false;   // gemv_i8 and its x order
  struct Regs {
    uint4 q[8];
    uint4 hdr;
    __half2 S[4], NM[4];   // tensor-core path: fp16 scale / negated-min pairs
    float sc[8], mb[8];    // GEMV path: fp32 scales and mins
  };
  static SW_DEVICE void load(const uint4* src, Regs& r) {
#pragma unroll
    for (int c = 0; c < 8; ++c) r.q[c] = src[c];
    r.hdr = src[8];
  }
  static SW_DEVICE void prep(Regs& r) { q4k_scales_h2(r.hdr, r.S, r.NM); }
  static SW_DEVICE void dq_chunk(const Regs& r, int c, uint32_t (&out)[16]) {
    dq_chunk_h2(r.q, r.S, r.NM, c, out);
  }
  static SW_DEVICE void gemv_prep(Regs& r) { q4k_scales_f32(r.hdr, r.sc, r.mb); }

  // Integer-dot variant of gemv (decode at 1..2 tokens): the activations of
  // the unit are quantized to int8 per 32 values (xq, built by quantize_x8
  // below), so 8 weights cost two nibble masks and two dp4a:
  //   sum_k (sc q_k - m) x_k ~= sc dx sum_k q_k xq_k - m dx sum_k xq_k.
  // The repacked nibble order puts K offsets (0,4,1,5) in the low nibbles
  // of a word's bytes and (2,6,3,7) in the high ones; quantize_x8 stores
  // the int8 activations in that order.
  template <int T>
  static SW_DEVICE void gemv_i8(const Regs& r, const uint2* xq, const float2* xs2,
                                float (&acc)[T]) {
    const uint32_t* qw = reinterpret_cast<const uint32_t*>(r.q);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      int is[T];
#pragma unroll
      for (int t = 0; t < T; ++t) is[t] = 0;
#pragma unroll
      for (int w4 = 0; w4 < 4; ++w4) {
        const uint32_t x = qw[4 * j + w4];
        const int lo = (int)(x & 0x0F0F0F0Fu), hi = (int)((x >> 4) & 0x0F0F0F0Fu);
#pragma unroll
        for (int t = 0; t < T; ++t) {
          const uint2 v = xq[t * 32 + 4 * j + w4];
          is[t] = __dp4a(lo, (int)v.x, is[t]);
          is[t] = __dp4a(hi, (int)v.y, is[t]);
        }
      }
#pragma unroll
      for (int t = 0; t < T; ++t) {
        const float2 dsum = xs2[t * 8 + j];   // (dx, sum of the rounded x) of sub-block j
        acc[t] = fmaf(r.sc[j] * dsum.x, (float)is[t], acc[t]);
        acc[t] = fmaf(-r.mb[j], dsum.y, acc[t]);
      }
    }
  }

  // The sub-block scale and min are applied once per 32 weights in fp32:
  //   sum_k (sc*q_k - m) x_k = sc * sum_k q_k x_k - m * sum_k x_k.
  // The fp16 partial sums hold 4 products each and are added in pairs (|sum|
  // <= 120 |x|max), so they stay finite for activations below ~500.
  template <int T>
  static SW_DEVICE void gemv(const Regs& r, const uint4* xs, float (&acc)[T], int lane) {
    const uint32_t MAGIC = 0x64006400u;
    const __half2 K1024 = u32_as_h2(0x64006400u);
    const __half2 SIXTEENTH = u32_as_h2(0x2C002C00u);   // 1/16, 1/16
    const __half2 M64 = u32_as_h2(0xD400D400u);         // -64, -64
    // sum_j m_j * (sum of x over sub-block j): lane l sums x[8l, 8l+8); four
    // lanes make a sub-block; every lane then needs all eight sub-block sums.
    float msum[T];
#pragma unroll
    for (int t = 0; t < T; ++t) {
      const uint4 v = xs[t * 32 + lane];
      const uint32_t vw[4] = {v.x, v.y, v.z, v.w};
      float s = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __half22float2(u32_as_h2(vw[e]));
        s += f.x + f.y;
      }
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      float m = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) m = fmaf(r.mb[j], __shfl_sync(0xffffffffu, s, 4 * j), m);
      msum[t] = m;
    }
    const uint32_t* qw = reinterpret_cast<const uint32_t*>(r.q);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      // four independent fp16 sums (one per nibble pair) keep the chains short
      __half2 p0[T], p1[T], p2[T], p3[T];
#pragma unroll
      for (int t = 0; t < T; ++t) p0[t] = p1[t] = p2[t] = p3[t] = __float2half2_rn(0.f);
#pragma unroll
      for (int w4 = 0; w4 < 4; ++w4) {
        const uint32_t xw = qw[4 * j + w4], hi = xw >> 8;
        // (k0,k1), (k2,k3), (k4,k5), (k6,k7) as exact fp16 integers
        const __half2 c0 = __hsub2(u32_as_h2(and_or(xw, 0x000F000Fu, MAGIC)), K1024);
        const __half2 c1 = __hfma2(u32_as_h2(and_or(xw, 0x00F000F0u, MAGIC)), SIXTEENTH, M64);
        const __half2 c2 = __hsub2(u32_as_h2(and_or(hi, 0x000F000Fu, MAGIC)), K1024);
        const __half2 c3 = __hfma2(u32_as_h2(and_or(hi, 0x00F000F0u, MAGIC)), SIXTEENTH, M64);
#pragma unroll
        for (int t = 0; t < T; ++t) {
          const uint4 xv = xs[t * 32 + 4 * j + w4];   // x[8w .. 8w+8) of this word
          p0[t] = __hfma2(c0, u32_as_h2(xv.x), p0[t]);
          p1[t] = __hfma2(c1, u32_as_h2(xv.y), p1[t]);
          p2[t] = __hfma2(c2, u32_as_h2(xv.z), p2[t]);
          p3[t] = __hfma2(c3, u32_as_h2(xv.w), p3[t]);
        }
      }
#pragma unroll
      for (int t = 0; t < T; ++t) {
        const float2 f0 = __half22float2(__hadd2(p0[t], p1[t]));
        const float2 f1 = __half22float2(__hadd2(p2[t], p3[t]));
        acc[t] = fmaf(r.sc[j], (f0.x + f0.y) + (f1.x + f1.y), acc[t]);
      }
    }
#pragma unroll
    for (int t = 0; t < T; ++t) acc[t] -= msum[t];
  }
};

// The activations of one 256-K unit as int8 for FmtQ4K::gemv_i8, built by the
// 32 lanes of a warp from the fp16 stage (lane l owns x[8l, 8l+8)): per 32
// values one scale dx = max|x| / 127 (round to nearest through the 1.5 * 2^23
// float trick), the int8 words in the repacked nibble order, and dx times the
// sum of the 32 rounded values.  The min term uses that sum of the rounded
// activations, so the result is exactly W . x_rounded: the rounding error is
// not multiplied by the (all-positive) scaled codes alone.
// xq: [T][32] uint2, xs2: [T][8] (dx, dx * sum).  NAT: the int8 words in
// plain K order ((0..3), (4..7)) instead, for formats with byte codes.
template <int T, bool NAT = false>
SW_DEVICE void quantize_x8(const uint4* xs, uint2* xq, float2* xs2, int lane) {
#pragma unroll
  for (int t = 0; t < T; ++t) {
    const uint4 v = xs[t * 32 + lane];
    const float2 f0 = __half22float2(u32_as_h2(v.x)), f1 = __half22float2(u32_as_h2(v.y));
    const float2 f2 = __half22float2(u32_as_h2(v.z)), f3 = __half22float2(u32_as_h2(v.w));
    // values k = 0..7 of this lane's word: (f0.x, f0.y, f1.x, f1.y, f2.x, f2.y, f3.x, f3.y)
    float amax = fmaxf(fmaxf(fmaxf(fabsf(f0.x), fabsf(f0.y)), fmaxf(fabsf(f1.x), fabsf(f1.y))),
                       fmaxf(fmaxf(fabsf(f2.x), fabsf(f2.y)), fmaxf(fabsf(f3.x), fabsf(f3.y))));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const float inv = amax > 0.f ? 127.f / amax : 0.f;
    const float M = 12582912.f;   // 1.5 * 2^23: the low mantissa byte is round(v) mod 256
    float sum = 0.f;
    auto q8 = [&](float x) {
      const float r = fmaf(x, inv, M);
      sum += r - M;               // the rounded value, exactly
      return (uint32_t)__float_as_int(r) & 0xFFu;
    };
    uint32_t lo, hi;
    if constexpr (NAT) {
      lo = q8(f0.x) | (q8(f0.y) << 8) | (q8(f1.x) << 16) | (q8(f1.y) << 24);
      hi = q8(f2.x) | (q8(f2.y) << 8) | (q8(f3.x) << 16) | (q8(f3.y) << 24);
    } else {
      // low-nibble partners: K (0, 4, 1, 5); high-nibble partners: K (2, 6, 3, 7)
      lo = q8(f0.x) | (q8(f2.x) << 8) | (q8(f0.y) << 16) | (q8(f2.y) << 24);
      hi = q8(f1.x) | (q8(f3.x) << 8) | (q8(f1.y) << 16) | (q8(f3.y) << 24);
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    xq[t * 32 + lane] = make_uint2(lo, hi);
    const float dx = amax * (1.f / 127.f);
    if ((lane & 3) == 0) xs2[t * 8 + (lane >> 2)] = make_float2(dx, dx * sum);
  }
}

// ----------------------------------------------------------------- Q6_K
constexpr int kQ6kRowBytes = 224;

// One low-nibble word x (K 8w..8w+7) and its crumbs h (pair j's at bits 2j,
// 16+2j) -> the four pairs (q - 32) as exact fp16 integers.  Pairs 1 and 3
// come out of the high nibble positions as 1024 + 16 q, which one HFMA2 by
// (1/16, -96) turns into q - 32 exactly.
SW_DEVICE void q6k_word(uint32_t x, uint32_t h, __half2 (&c)[4]) {
  const uint32_t MAGIC = 0x64006400u;
  const __half2 K1056 = u32_as_h2(0x64206420u);        // 1056 = 1024 + 32
  const __half2 SIXTEENTH = u32_as_h2(0x2C002C00u);
  const __half2 M96 = u32_as_h2(0xD600D600u);          // -96
  const uint32_t hi = x >> 8;
  c[0] = __hsub2(u32_as_h2(and_or(h << 4, 0x00300030u, and_or(x, 0x000F000Fu, MAGIC))), K1056);
  c[1] = __hfma2(u32_as_h2(and_or(h << 6, 0x03000300u, and_or(x, 0x00F000F0u, MAGIC))),
                 SIXTEENTH, M96);
  c[2] = __hsub2(u32_as_h2(and_or(h, 0x00300030u, and_or(hi, 0x000F000Fu, MAGIC))), K1056);
  c[3] = __hfma2(u32_as_h2(and_or(h << 2, 0x03000300u, and_or(hi, 0x00F000F0u, MAGIC))),
                 SIXTEENTH, M96);
}

struct FmtQ6K {
  static constexpr int ID = kFmtQ6K;
  static constexpr int ROW_BYTES = kQ6kRowBytes;
  static constexpr bool HAS_I8 = true, X8_NATURAL = false;
  struct Regs {
    uint4 lo[8];   // 32 low-nibble words
    uint4 hc[4];   // 16 crumb words
    uint4 sc[2];   // 16 fp16 scales
  };
  static SW_DEVICE void load(const uint4* src, Regs& r) {
#pragma unroll
    for (int c = 0; c < 8; ++c) r.lo[c] = src[c];
#pragma unroll
    for (int c = 0; c < 4; ++c) r.hc[c] = src[8 + c];
    r.sc[0] = src[12];
    r.sc[1] = src[13];
  }
  static SW_DEVICE void prep(Regs&) {}
  static SW_DEVICE void gemv_prep(Regs&) {}
  static SW_DEVICE void dq_chunk(const Regs& r, int sp, uint32_t (&cols)[16]) {
    const uint32_t* lw = reinterpret_cast<const uint32_t*>(r.lo);
    const uint32_t* hw = reinterpret_cast<const uint32_t*>(r.hc);
    const uint32_t* sw = reinterpret_cast<const uint32_t*>(r.sc);   // scale pairs (2s, 2s+1)
    {                                         // two sub-blocks = 32 K = 16 columns
      const __half2 s2 = u32_as_h2(sw[sp]);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int s = 2 * sp + half;
        const __half2 S = half ? __high2half2(s2) : __low2half2(s2);
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          __half2 c[4];
          q6k_word(lw[2 * s + e], e ? hw[s] >> 8 : hw[s], c);
#pragma unroll
          for (int j = 0; j < 4; ++j) cols[8 * half + 4 * e + j] = h2_as_u32(__hmul2(c[j], S));
        }
      }
    }
  }
  // Integer-dot variant: the 6-bit codes of a word rebuilt as bytes in the
  // repacked nibble order (low nibble | crumb << 4: the crumbs of K' = 0, 4,
  // 1, 5 sit at bits 0, 4, 16, 20 of the crumb word, those of 2, 6, 3, 7 two
  // bits higher), minus 32 per byte, then dp4a against the int8 activations;
  // the fp16 sub-block scale (16 values) times the activation scale (32
  // values) in fp32.
  template <int T>
  static SW_DEVICE void gemv_i8(const Regs& r, const uint2* xq, const float2* xs2,
                                float (&acc)[T]) {
    const uint32_t* lw = reinterpret_cast<const uint32_t*>(r.lo);
    const uint32_t* hw = reinterpret_cast<const uint32_t*>(r.hc);
    const __half* sh = reinterpret_cast<const __half*>(r.sc);
#pragma unroll
    for (int s = 0; s < 16; ++s) {
      int is[T];
#pragma unroll
      for (int t = 0; t < T; ++t) is[t] = 0;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const uint32_t x = lw[2 * s + e], h = e ? hw[s] >> 8 : hw[s];
        const uint32_t lo = and_or(h << 8, 0x30003000u,
                                   and_or(h << 4, 0x00300030u, x & 0x0F0F0F0Fu));
        const uint32_t hi = and_or(h << 6, 0x30003000u,
                                   and_or(h << 2, 0x00300030u, (x >> 4) & 0x0F0F0F0Fu));
        const int slo = (int)__vsub4(lo, 0x20202020u), shi = (int)__vsub4(hi, 0x20202020u);
#pragma unroll
        for (int t = 0; t < T; ++t) {
          const uint2 v = xq[t * 32 + 2 * s + e];
          is[t] = __dp4a(slo, (int)v.x, is[t]);
          is[t] = __dp4a(shi, (int)v.y, is[t]);
        }
      }
      const float S = __half2float(sh[s]);
#pragma unroll
      for (int t = 0; t < T; ++t) acc[t] = fmaf(S * xs2[t * 8 + (s >> 1)].x, (float)is[t], acc[t]);
    }
  }

  // (q - 32) x products in fp16: two per partial sum (|sum| <= 64 |x|max),
  // then the sub-block scale in fp32.
  template <int T>
  static SW_DEVICE void gemv(const Regs& r, const uint4* xs, float (&acc)[T], int) {
    const uint32_t* lw = reinterpret_cast<const uint32_t*>(r.lo);
    const uint32_t* hw = reinterpret_cast<const uint32_t*>(r.hc);
    const __half* sh = reinterpret_cast<const __half*>(r.sc);
#pragma unroll
    for (int s = 0; s < 16; ++s) {
      __half2 p[4][T];
#pragma unroll
      for (int t = 0; t < T; ++t) p[0][t] = p[1][t] = p[2][t] = p[3][t] = __float2half2_rn(0.f);
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        __half2 c[4];
        q6k_word(lw[2 * s + e], e ? hw[s] >> 8 : hw[s], c);
#pragma unroll
        for (int t = 0; t < T; ++t) {
          const uint4 xv = xs[t * 32 + 2 * s + e];
          p[0][t] = __hfma2(c[0], u32_as_h2(xv.x), p[0][t]);
          p[1][t] = __hfma2(c[1], u32_as_h2(xv.y), p[1][t]);
          p[2][t] = __hfma2(c[2], u32_as_h2(xv.z), p[2][t]);
          p[3][t] = __hfma2(c[3], u32_as_h2(xv.w), p[3][t]);
        }
      }
      const float S = __half2float(sh[s]);
#pragma unroll
      for (int t = 0; t < T; ++t) {
        const float2 f0 = __half22float2(p[0][t]), f1 = __half22float2(p[1][t]);
        const float2 f2 = __half22float2(p[2][t]), f3 = __half22float2(p[3][t]);
        acc[t] = fmaf(S, ((f0.x + f0.y) + (f1.x + f1.y)) + ((f2.x + f2.y) + (f3.x + f3.y)),
                      acc[t]);
      }
    }
  }
};

// ----------------------------------------------------------------- Q8_0
constexpr int kQ80RowBytes = 272;

// Code word (4 unsigned codes u = q + 128, K order) -> pairs (k0,k1), (k2,k3)
// of q * d: a byte permute places u under the 0x64 exponent byte (1024 + u),
// minus 1152 gives q exactly, and one multiply applies the block scale.
SW_DEVICE void q80_word(uint32_t x, __half2 D, uint32_t* out) {
  const __half2 K1152 = u32_as_h2(0x64806480u);   // 1152 = 1024 + 128
  out[0] = h2_as_u32(__hmul2(__hsub2(u32_as_h2(byte_perm(x, 0x64646464u, 0x5140u)), K1152), D));
  out[1] = h2_as_u32(__hmul2(__hsub2(u32_as_h2(byte_perm(x, 0x64646464u, 0x5342u)), K1152), D));
}

struct FmtQ80 {
  static constexpr int ID = kFmtQ8_0;
  static constexpr int ROW_BYTES = kQ80RowBytes;
  static constexpr bool HAS_I8 = true, X8_NATURAL = true;
  struct Regs {
    uint4 q[16];   // 64 code words
    uint4 d;       // 8 fp16 block scales
  };
  static SW_DEVICE void load(const uint4* src, Regs& r) {
#pragma unroll
    for (int c = 0; c < 16; ++c) r.q[c] = src[c];
    r.d = src[16];
  }
  static SW_DEVICE void prep(Regs&) {}
  static SW_DEVICE void gemv_prep(Regs&) {}
  static SW_DEVICE void dq_chunk(const Regs& r, int b, uint32_t (&out)[16]) {
    const uint32_t* qw = reinterpret_cast<const uint32_t*>(r.q);
    const uint32_t* dw = reinterpret_cast<const uint32_t*>(&r.d);
    const __half2 d2 = u32_as_h2(dw[b >> 1]);   // one 32-value block = 16 columns
    const __half2 D = (b & 1) ? __high2half2(d2) : __low2half2(d2);
#pragma unroll
    for (int w = 0; w < 8; ++w) q80_word(qw[8 * b + w], D, out + 2 * w);
  }
  // Integer-dot variant (activations quantized per 32 values in plain K
  // order): per 32-value block 8 dp4a of the signed codes (u ^ 0x80) and the
  // int8 activations, then d * dx in fp32.
  template <int T>
  static SW_DEVICE void gemv_i8(const Regs& r, const uint2* xq, const float2* xs2,
                                float (&acc)[T]) {
    const uint32_t* qw = reinterpret_cast<const uint32_t*>(r.q);
    const __half* dh = reinterpret_cast<const __half*>(&r.d);
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      int is[T];
#pragma unroll
      for (int t = 0; t < T; ++t) is[t] = 0;
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        const int c0 = (int)(qw[8 * b + 2 * v] ^ 0x80808080u);
        const int c1 = (int)(qw[8 * b + 2 * v + 1] ^ 0x80808080u);
#pragma unroll
        for (int t = 0; t < T; ++t) {
          const uint2 xv = xq[t * 32 + 4 * b + v];
          is[t] = __dp4a(c0, (int)xv.x, is[t]);
          is[t] = __dp4a(c1, (int)xv.y, is[t]);
        }
      }
      const float d = __half2float(dh[b]);
#pragma unroll
      for (int t = 0; t < T; ++t) acc[t] = fmaf(d * xs2[t * 8 + b].x, (float)is[t], acc[t]);
    }
  }

  // Weights are scaled before the products (q*d is what the tensor-core path
  // multiplies too), so the fp16 partials hold ordinary w*x sums.
  template <int T>
  static SW_DEVICE void gemv(const Regs& r, const uint4* xs, float (&acc)[T], int) {
    const uint32_t* qw = reinterpret_cast<const uint32_t*>(r.q);
    const uint32_t* dw = reinterpret_cast<const uint32_t*>(&r.d);
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      const __half2 d2 = u32_as_h2(dw[b >> 1]);
      const __half2 D = (b & 1) ? __high2half2(d2) : __low2half2(d2);
      __half2 p[4][T];
#pragma unroll
      for (int t = 0; t < T; ++t) p[0][t] = p[1][t] = p[2][t] = p[3][t] = __float2half2_rn(0.f);
#pragma unroll
      for (int v = 0; v < 4; ++v) {           // x uint4 = 8 values = 2 code words
        uint32_t c[4];
        q80_word(qw[8 * b + 2 * v], D, c);
        q80_word(qw[8 * b + 2 * v + 1], D, c + 2);
#pragma unroll
        for (int t = 0; t < T; ++t) {
          const uint4 xv = xs[t * 32 + 4 * b + v];
          p[0][t] = __hfma2(u32_as_h2(c[0]), u32_as_h2(xv.x), p[0][t]);
          p[1][t] = __hfma2(u32_as_h2(c[1]), u32_as_h2(xv.y), p[1][t]);
          p[2][t] = __hfma2(u32_as_h2(c[2]), u32_as_h2(xv.z), p[2][t]);
          p[3][t] = __hfma2(u32_as_h2(c[3]), u32_as_h2(xv.w), p[3][t]);
        }
      }
#pragma unroll
      for (int t = 0; t < T; ++t) {
        const float2 f0 = __half22float2(__hadd2(p[0][t], p[1][t]));
        const float2 f1 = __half22float2(__hadd2(p[2][t], p[3][t]));
        acc[t] += (f0.x + f0.y) + (f1.x + f1.y);
      }
    }
  }
};

}  // namespace swarm
