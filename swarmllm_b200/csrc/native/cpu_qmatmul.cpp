// Quantized matmul on the host CPU: out[t][r] = sum_k W[r][k] * x[t][k] with W
// in its GGUF blocks (Q4_K, Q6_K, Q8_0, Q4_0, IQ4_NL, IQ4_XS, MXFP4), never
// dequantized to a float matrix.
//
// The activations of every token are quantized once per call to int8 with one
// scale per 32 values (absmax / 127, round to nearest), and each block's dot
// product is an int8 x int8 -> int32 loop the compiler vectorises; the block
// and sub-block scales are applied in fp32:
//   Q8_0  sum_b d_b dx_b sum q x
//   Q4_0  sum_b d_b dx_b sum (q - 8) x
//   IQ4_NL / MXFP4  sum_b s_b dx_b sum book[q] x  (s_b: fp16 d, or 2^(e - 128))
//   IQ4_XS  sum_j d (ls_j - 32) dx_j sum book[q] x  (32-value sub-blocks)
//   Q6_K  sum_s d sc_s dx sum (q - 32) x                (16-value sub-blocks)
//   Q4_K  sum_j d sc_j dx_j sum q x - dmin m_j dx_j sum x  (32-value sub-blocks)
// with the min term over the rounded activations, so the result is exactly
// W . x_rounded.  Rows are split over OpenMP threads.
//
// On CPUs with AVX-512 VNNI (picked at run time) the codes of each 64-value
// group go through one vpdpbusd (unsigned codes x signed activations, four
// products per 32-bit lane) per token; a lane's partial sum is scaled in fp32
// by its sub-block's scale times its activation block's scale, so all three
// formats share one inner loop and differ only in how a block is unpacked:
// Q4_K and Q4_0 codes are already unsigned (Q4_0 before its -8), Q6_K codes
// are used before their -32 and Q8_0 codes are flipped to q + 128; the
// offsets come back as one correction per block against the sums of the
// rounded activations.  This is the CPU
// inference path of a node without a GPU (the reference's CPU kernels:
// src/inference/split/attn_rows.rs, fast_math.rs); the fp32 PyTorch model
// stays the numerical oracle.
#include "cpu_qmatmul.h"

#include <immintrin.h>

#include <cmath>
#include <cstdlib>
#include <cstring>
#include <vector>

namespace swarm_native {
namespace {

inline float half_to_float(uint16_t h) {
  const uint32_t s = (uint32_t)(h >> 15) << 31;
  uint32_t e = (h >> 10) & 0x1F, m = h & 0x3FF;
  uint32_t bits;
  if (e == 0) {
    if (m == 0) {
      bits = s;
    } else {  // subnormal: normalise
      e = 127 - 15 + 1;
      while (!(m & 0x400)) {
        m <<= 1;
        --e;
      }
      bits = s | (e << 23) | ((m & 0x3FF) << 13);
    }
  } else if (e == 31) {
    bits = s | 0x7F800000u | (m << 13);
  } else {
    bits = s | ((e + 127 - 15) << 23) | (m << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

// x [K] -> int8 [K], dx [K/32] scales, sx [K/32] sums of the rounded values
void quantize_row(const float* x, int K, int8_t* q, float* dx, int32_t* sx) {
  for (int b = 0; b < K / 32; ++b) {
    const float* xb = x + 32 * b;
    float amax = 0.f;
    for (int i = 0; i < 32; ++i) amax = std::fmax(amax, std::fabs(xb[i]));
    const float inv = amax > 0.f ? 127.f / amax : 0.f;
    int32_t s = 0;
    for (int i = 0; i < 32; ++i) {
      const int v = (int)std::nearbyint(xb[i] * inv);
      q[32 * b + i] = (int8_t)v;
      s += v;
    }
    dx[b] = amax / 127.f;
    sx[b] = s;
  }
}

inline int32_t dot_i8(const int8_t* a, const int8_t* b, int n) {
  int32_t s = 0;
  for (int i = 0; i < n; ++i) s += (int32_t)a[i] * (int32_t)b[i];
  return s;
}

// Token tile: a block's codes are unpacked once and dotted with this many
// tokens' activations before the next block.
constexpr int kTT = 8;

struct Acts {
  const int8_t* q;    // [T, K]
  const float* dx;    // [T, K/32]
  const int32_t* sx;  // [T, K/32]
  int K;
};

// The 4-bit code books of the table formats (value = scale * code).
constexpr int8_t kIq4Code[16] = {-127, -104, -83, -65, -49, -35, -22, -10,
                                 1,    13,   25,  38,  53,  69,  89,  113};
// MXFP4: E2M1 values doubled (0, 0.5, ..., 6 -> 0, 1, ..., 12); the E8M0 block
// scale 2^(e - 128) then gives the value.
constexpr int8_t kMxfp4Code[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};

// Block scale of a table format: fp16 d (IQ4_NL) or E8M0 exponent (MXFP4).
inline float lut_scale(int type, const uint8_t* blk) {
  return type == kGgmlIQ4_NL ? half_to_float(rd16(blk)) : std::ldexp(1.f, (int)blk[0] - 128);
}

// IQ4_XS sub-block scales: d * (ls_j - 32), ls_j six bits (4 low in
// scales_l, 2 high in scales_h).
inline void iq4xs_scales(const uint8_t* blk, float* dl) {
  const float d = half_to_float(rd16(blk));
  const int sh = rd16(blk + 2);
  for (int j = 0; j < 8; ++j) {
    const int ls = ((blk[4 + j / 2] >> (4 * (j % 2))) & 0xF) | (((sh >> (2 * j)) & 3) << 4);
    dl[j] = d * (float)(ls - 32);
  }
}

// One block decoded to integer codes and per-sub-block affine maps:
// value[i] = scale[i / sub] * q[i] + offset[i / sub].
struct Decoded {
  int8_t q[256];
  float scale[16], offset[16];
  int n, sub;  // values in the block, values per sub-block
};

void decode_block(int type, const uint8_t* blk, Decoded& o) {
  switch (type) {
    case kGgmlQ4_K: {
      const float d = half_to_float(rd16(blk)), dmin = half_to_float(rd16(blk + 2));
      const uint8_t* sc = blk + 4;
      const uint8_t* qs = blk + 16;
      for (int g = 0; g < 4; ++g)
        for (int l = 0; l < 32; ++l) {
          o.q[64 * g + l] = (int8_t)(qs[32 * g + l] & 0xF);
          o.q[64 * g + 32 + l] = (int8_t)(qs[32 * g + l] >> 4);
        }
      for (int j = 0; j < 8; ++j) {
        int sv, m;
        if (j < 4) {
          sv = sc[j] & 63;
          m = sc[j + 4] & 63;
        } else {
          sv = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
          m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
        }
        o.scale[j] = d * (float)sv;
        o.offset[j] = -dmin * (float)m;
      }
      o.n = 256;
      o.sub = 32;
      return;
    }
    case kGgmlQ6_K: {
      const uint8_t* ql = blk;
      const uint8_t* qh = blk + 128;
      const int8_t* sc = reinterpret_cast<const int8_t*>(blk + 192);
      const float d = half_to_float(rd16(blk + 208));
      for (int n = 0; n < 2; ++n)
        for (int l = 0; l < 32; ++l) {
          const int h = qh[32 * n + l];
          const int l0 = ql[64 * n + l], l1 = ql[64 * n + 32 + l];
          o.q[128 * n + l] = (int8_t)(((l0 & 0xF) | ((h & 3) << 4)) - 32);
          o.q[128 * n + 32 + l] = (int8_t)(((l1 & 0xF) | (((h >> 2) & 3) << 4)) - 32);
          o.q[128 * n + 64 + l] = (int8_t)(((l0 >> 4) | (((h >> 4) & 3) << 4)) - 32);
          o.q[128 * n + 96 + l] = (int8_t)(((l1 >> 4) | (((h >> 6) & 3) << 4)) - 32);
        }
      for (int j = 0; j < 16; ++j) {
        o.scale[j] = d * (float)sc[j];
        o.offset[j] = 0.f;
      }
      o.n = 256;
      o.sub = 16;
      return;
    }
    case kGgmlIQ4_XS: {
      iq4xs_scales(blk, o.scale);
      for (int j = 0; j < 8; ++j) {
        o.offset[j] = 0.f;
        for (int i = 0; i < 16; ++i) {
          const uint8_t c = blk[8 + 16 * j + i];
          o.q[32 * j + i] = kIq4Code[c & 0xF];
          o.q[32 * j + 16 + i] = kIq4Code[c >> 4];
        }
      }
      o.n = 256;
      o.sub = 32;
      return;
    }
    case kGgmlQ8_0: {
      o.scale[0] = half_to_float(rd16(blk));
      std::memcpy(o.q, blk + 2, 32);
      break;
    }
    default: {  // Q4_0, IQ4_NL, MXFP4: 32 codes in the nibbles of 16 bytes
      const int hdr = type == kGgmlMXFP4 ? 1 : 2;
      o.scale[0] = type == kGgmlQ4_0 ? half_to_float(rd16(blk)) : lut_scale(type, blk);
      for (int j = 0; j < 16; ++j) {
        const uint8_t c = blk[hdr + j];
        if (type == kGgmlQ4_0) {
          o.q[j] = (int8_t)((c & 0xF) - 8);
          o.q[16 + j] = (int8_t)((c >> 4) - 8);
        } else {
          const int8_t* book = type == kGgmlIQ4_NL ? kIq4Code : kMxfp4Code;
          o.q[j] = book[c & 0xF];
          o.q[16 + j] = book[c >> 4];
        }
      }
      break;
    }
  }
  o.offset[0] = 0.f;
  o.n = 32;
  o.sub = 32;
}

// One block of any format against tokens t0..t0+nt (the portable path).
// A sub-block's activation scale is the one of its 32-value activation
// block; an offset (Q4_K's -dmin m) meets the sum of the rounded activations.
void block_generic(int type, const uint8_t* blk, int vpos, const Acts& a, int t0, int nt,
                   float* acc) {
  Decoded o;
  decode_block(type, blk, o);
  const int nb = a.K / 32, ns = o.n / o.sub;
  for (int t = 0; t < nt; ++t) {
    const int8_t* xq = a.q + (size_t)(t0 + t) * a.K + vpos;
    const float* dx = a.dx + (size_t)(t0 + t) * nb + vpos / 32;
    const int32_t* sx = a.sx + (size_t)(t0 + t) * nb + vpos / 32;
    float v = 0.f;
    for (int j = 0; j < ns; ++j) {
      const int x32 = j * o.sub / 32;
      v += o.scale[j] * dx[x32] * (float)dot_i8(o.q + j * o.sub, xq + j * o.sub, o.sub);
      if (o.offset[j] != 0.f) v += o.offset[j] * dx[x32] * (float)sx[x32];
    }
    acc[t] += v;
  }
}

size_t row_bytes_of(int type, int K) {
  switch (type) {
    case kGgmlQ4_K: return (size_t)K / 256 * 144;
    case kGgmlQ6_K: return (size_t)K / 256 * 210;
    case kGgmlQ8_0: return (size_t)K / 32 * 34;
    case kGgmlMXFP4: return (size_t)K / 32 * 17;
    case kGgmlIQ4_XS: return (size_t)K / 256 * 136;
    default: return (size_t)K / 32 * 18;  // Q4_0, IQ4_NL
  }
}

// ---------------------------------------------------------------- AVX-512 VNNI
#define SWARM_VNNI __attribute__((target("avx512f,avx512bw,avx512dq,avx512vl,avx512vnni")))

// Lane i of a 64-value group g holds values 64g + 4i .. 64g + 4i + 3, whose
// activation block is 2g + (i >= 8).
struct ActsX {
  const int8_t* q;      // [T, K]
  const float* dx;      // [T, K/32]
  const float* dxs;     // [T, K/32]: dx * (sum of the rounded values), per 32
  const float* dxs16;   // [T, K/16]: dx * (sum of the rounded values), per 16
  int K;
};

// One 256-value block unpacked for the shared loop: unsigned codes of the four
// 64-value groups, the per-lane weight scales, and the offset correction
// `corr` dotted with the activation sums (8 per-32 sums, or 16 per-16 sums).
struct Unpacked {
  __m512i c[4];
  __m512 s[4];
  __m512 corr;  // Q6_K: 16 lanes; Q4_K / Q8_0: lanes 0-7
};

SWARM_VNNI inline __m512 halves(float a, float b) {
  return _mm512_insertf32x8(_mm512_castps256_ps512(_mm256_set1_ps(a)), _mm256_set1_ps(b), 1);
}

SWARM_VNNI inline void unpack_q4k(const uint8_t* blk, Unpacked& u) {
  const float d = half_to_float(rd16(blk)), dmin = half_to_float(rd16(blk + 2));
  const uint8_t* sc = blk + 4;
  const uint8_t* qs = blk + 16;
  float ds[8], dm[8];
  for (int j = 0; j < 8; ++j) {
    int s, m;
    if (j < 4) {
      s = sc[j] & 63;
      m = sc[j + 4] & 63;
    } else {
      s = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
      m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
    }
    ds[j] = d * (float)s;
    dm[j] = dmin * (float)m;
  }
  const __m256i lo4 = _mm256_set1_epi8(0x0F);
  for (int g = 0; g < 4; ++g) {
    const __m256i v = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(qs + 32 * g));
    const __m256i lo = _mm256_and_si256(v, lo4);
    const __m256i hi = _mm256_and_si256(_mm256_srli_epi16(v, 4), lo4);
    u.c[g] = _mm512_inserti64x4(_mm512_castsi256_si512(lo), hi, 1);
    u.s[g] = halves(ds[2 * g], ds[2 * g + 1]);
  }
  u.corr = _mm512_castps256_ps512(_mm256_loadu_ps(dm));
}

// bits sh, sh+1 of every qh byte, moved to bits 4-5
SWARM_VNNI inline __m256i q6_hi(__m256i h, int sh, __m256i two) {
  return _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(h, sh), two), 4);
}

SWARM_VNNI inline void unpack_q6k(const uint8_t* blk, Unpacked& u) {
  const uint8_t* ql = blk;
  const uint8_t* qh = blk + 128;
  const int8_t* sc = reinterpret_cast<const int8_t*>(blk + 192);
  const float d = half_to_float(rd16(blk + 208));
  alignas(64) float ds[16];
  for (int i = 0; i < 16; ++i) ds[i] = d * (float)sc[i];
  const __m256i lo4 = _mm256_set1_epi8(0x0F), two = _mm256_set1_epi8(0x03);
  for (int n = 0; n < 2; ++n) {
    const __m256i l0 = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(ql + 64 * n));
    const __m256i l1 = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(ql + 64 * n + 32));
    const __m256i h = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(qh + 32 * n));
    const __m256i q0 = _mm256_or_si256(_mm256_and_si256(l0, lo4), q6_hi(h, 0, two));
    const __m256i q1 = _mm256_or_si256(_mm256_and_si256(l1, lo4), q6_hi(h, 2, two));
    const __m256i q2 =
        _mm256_or_si256(_mm256_and_si256(_mm256_srli_epi16(l0, 4), lo4), q6_hi(h, 4, two));
    const __m256i q3 =
        _mm256_or_si256(_mm256_and_si256(_mm256_srli_epi16(l1, 4), lo4), q6_hi(h, 6, two));
    u.c[2 * n] = _mm512_inserti64x4(_mm512_castsi256_si512(q0), q1, 1);
    u.c[2 * n + 1] = _mm512_inserti64x4(_mm512_castsi256_si512(q2), q3, 1);
  }
  // lane i of group g covers values 64g + 4i..: sub-block 4g + i / 4
  const __m512i rep4 = _mm512_set_epi32(3, 3, 3, 3, 2, 2, 2, 2, 1, 1, 1, 1, 0, 0, 0, 0);
  for (int g = 0; g < 4; ++g)
    u.s[g] = _mm512_permutexvar_ps(rep4, _mm512_castps128_ps512(_mm_loadu_ps(ds + 4 * g)));
  u.corr = _mm512_mul_ps(_mm512_load_ps(ds), _mm512_set1_ps(32.f));
}

// Eight Q8_0 blocks (256 values, 8 x 34 bytes), codes flipped to q + 128.
SWARM_VNNI inline void unpack_q80x8(const uint8_t* blk, Unpacked& u) {
  float d[8];
  const __m256i flip = _mm256_set1_epi8((char)0x80);
  for (int j = 0; j < 8; ++j) d[j] = half_to_float(rd16(blk + 34 * j));
  for (int g = 0; g < 4; ++g) {
    const __m256i a = _mm256_xor_si256(
        _mm256_loadu_si256(reinterpret_cast<const __m256i*>(blk + 34 * (2 * g) + 2)), flip);
    const __m256i b = _mm256_xor_si256(
        _mm256_loadu_si256(reinterpret_cast<const __m256i*>(blk + 34 * (2 * g + 1) + 2)), flip);
    u.c[g] = _mm512_inserti64x4(_mm512_castsi256_si512(a), b, 1);
    u.s[g] = halves(d[2 * g], d[2 * g + 1]);
  }
  u.corr = _mm512_mul_ps(_mm512_castps256_ps512(_mm256_loadu_ps(d)), _mm512_set1_ps(128.f));
}

// Eight Q4_0 blocks (256 values, 8 x 18 bytes): the codes as they are (0..15),
// the offset of 8 back through the correction.
SWARM_VNNI inline void unpack_q40x8(const uint8_t* blk, Unpacked& u) {
  float d[8];
  const __m128i lo4 = _mm_set1_epi8(0x0F);
  for (int j = 0; j < 8; ++j) d[j] = half_to_float(rd16(blk + 18 * j));
  for (int g = 0; g < 4; ++g) {
    __m256i half[2];
    for (int h = 0; h < 2; ++h) {
      const __m128i v = _mm_loadu_si128(reinterpret_cast<const __m128i*>(blk + 18 * (2 * g + h) + 2));
      const __m128i lo = _mm_and_si128(v, lo4);
      const __m128i hi = _mm_and_si128(_mm_srli_epi16(v, 4), lo4);
      half[h] = _mm256_inserti128_si256(_mm256_castsi128_si256(lo), hi, 1);
    }
    u.c[g] = _mm512_inserti64x4(_mm512_castsi256_si512(half[0]), half[1], 1);
    u.s[g] = halves(d[2 * g], d[2 * g + 1]);
  }
  u.corr = _mm512_mul_ps(_mm512_castps256_ps512(_mm256_loadu_ps(d)), _mm512_set1_ps(8.f));
}

// Eight IQ4_NL / MXFP4 blocks: each nibble looked up (pshufb) in the code
// book shifted by +128, so the codes are unsigned; the +128 comes back through
// the correction as for Q8_0.
template <int TYPE>
SWARM_VNNI inline void unpack_lut4x8(const uint8_t* blk, Unpacked& u) {
  constexpr int BB = TYPE == kGgmlIQ4_NL ? 18 : 17, HDR = TYPE == kGgmlIQ4_NL ? 2 : 1;
  const int8_t* book = TYPE == kGgmlIQ4_NL ? kIq4Code : kMxfp4Code;
  alignas(16) uint8_t ub[16];
  for (int i = 0; i < 16; ++i) ub[i] = (uint8_t)(book[i] + 128);
  const __m128i table = _mm_load_si128(reinterpret_cast<const __m128i*>(ub));
  const __m128i lo4 = _mm_set1_epi8(0x0F);
  float d[8];
  for (int j = 0; j < 8; ++j) d[j] = lut_scale(TYPE, blk + BB * j);
  for (int g = 0; g < 4; ++g) {
    __m256i half[2];
    for (int h = 0; h < 2; ++h) {
      const __m128i v = _mm_loadu_si128(reinterpret_cast<const __m128i*>(blk + BB * (2 * g + h) + HDR));
      const __m128i lo = _mm_shuffle_epi8(table, _mm_and_si128(v, lo4));
      const __m128i hi = _mm_shuffle_epi8(table, _mm_and_si128(_mm_srli_epi16(v, 4), lo4));
      half[h] = _mm256_inserti128_si256(_mm256_castsi128_si256(lo), hi, 1);
    }
    u.c[g] = _mm512_inserti64x4(_mm512_castsi256_si512(half[0]), half[1], 1);
    u.s[g] = halves(d[2 * g], d[2 * g + 1]);
  }
  u.corr = _mm512_mul_ps(_mm512_castps256_ps512(_mm256_loadu_ps(d)), _mm512_set1_ps(128.f));
}

// One IQ4_XS block: its eight sub-blocks through the IQ4 code book (+128).
SWARM_VNNI inline void unpack_iq4xs(const uint8_t* blk, Unpacked& u) {
  alignas(16) uint8_t ub[16];
  for (int i = 0; i < 16; ++i) ub[i] = (uint8_t)(kIq4Code[i] + 128);
  const __m128i table = _mm_load_si128(reinterpret_cast<const __m128i*>(ub));
  const __m128i lo4 = _mm_set1_epi8(0x0F);
  float dl[8];
  iq4xs_scales(blk, dl);
  for (int g = 0; g < 4; ++g) {
    __m256i half[2];
    for (int h = 0; h < 2; ++h) {
      const __m128i v =
          _mm_loadu_si128(reinterpret_cast<const __m128i*>(blk + 8 + 16 * (2 * g + h)));
      const __m128i lo = _mm_shuffle_epi8(table, _mm_and_si128(v, lo4));
      const __m128i hi = _mm_shuffle_epi8(table, _mm_and_si128(_mm_srli_epi16(v, 4), lo4));
      half[h] = _mm256_inserti128_si256(_mm256_castsi128_si256(lo), hi, 1);
    }
    u.c[g] = _mm512_inserti64x4(_mm512_castsi256_si512(half[0]), half[1], 1);
    u.s[g] = halves(dl[2 * g], dl[2 * g + 1]);
  }
  u.corr = _mm512_mul_ps(_mm512_castps256_ps512(_mm256_loadu_ps(dl)), _mm512_set1_ps(128.f));
}

// out[t] for tokens t0..t0+nt of one weight row; FMT 0 Q4_K, 1 Q6_K, 2 Q8_0,
// 3 Q4_0, 4 IQ4_NL, 5 MXFP4, 6 IQ4_XS.
template <int FMT>
SWARM_VNNI void row_vnni(const uint8_t* wr, int nsb, const ActsX& a, int t0, int nt, float* res) {
  constexpr size_t SB_BYTES = FMT == 0   ? 144
                              : FMT == 6 ? 136
                              : FMT == 1 ? 210
                              : FMT == 2 ? 8 * 34
                              : FMT == 5 ? 8 * 17
                                         : 8 * 18;
  __m512 facc[kTT], cacc[kTT];
  for (int t = 0; t < nt; ++t) facc[t] = cacc[t] = _mm512_setzero_ps();
  // lanes 0-7 take the group's first activation scale, lanes 8-15 its second
  const __m512i pair = _mm512_set_epi32(1, 1, 1, 1, 1, 1, 1, 1, 0, 0, 0, 0, 0, 0, 0, 0);
  const int K = a.K;
  for (int b = 0; b < nsb; ++b) {
    Unpacked u;
    if constexpr (FMT == 0) unpack_q4k(wr + b * SB_BYTES, u);
    else if constexpr (FMT == 1) unpack_q6k(wr + b * SB_BYTES, u);
    else if constexpr (FMT == 2) unpack_q80x8(wr + b * SB_BYTES, u);
    else if constexpr (FMT == 3) unpack_q40x8(wr + b * SB_BYTES, u);
    else if constexpr (FMT == 4) unpack_lut4x8<kGgmlIQ4_NL>(wr + b * SB_BYTES, u);
    else if constexpr (FMT == 5) unpack_lut4x8<kGgmlMXFP4>(wr + b * SB_BYTES, u);
    else unpack_iq4xs(wr + b * SB_BYTES, u);
    for (int t = 0; t < nt; ++t) {
      const size_t tt = (size_t)(t0 + t);
      const int8_t* xq = a.q + tt * K + 256 * b;
      const float* dx = a.dx + tt * (K / 32) + 8 * b;
      __m512 f = facc[t];
      for (int g = 0; g < 4; ++g) {
        const __m512i xv = _mm512_loadu_si512(xq + 64 * g);
        const __m512i p = _mm512_dpbusd_epi32(_mm512_setzero_si512(), u.c[g], xv);
        const __m512 dxg = _mm512_permutexvar_ps(
            pair, _mm512_castpd_ps(_mm512_castpd128_pd512(_mm_load_sd(reinterpret_cast<const double*>(dx + 2 * g)))));
        const __m512 sc = _mm512_mul_ps(u.s[g], dxg);
        f = _mm512_fmadd_ps(_mm512_cvtepi32_ps(p), sc, f);
      }
      facc[t] = f;
      const __m512 sums = FMT == 1 ? _mm512_loadu_ps(a.dxs16 + tt * (K / 16) + 16 * b)
                                   : _mm512_castps256_ps512(_mm256_loadu_ps(a.dxs + tt * (K / 32) + 8 * b));
      const __m512 cm = FMT == 1 ? u.corr : _mm512_maskz_mov_ps(0x00FF, u.corr);
      cacc[t] = _mm512_fmadd_ps(cm, _mm512_maskz_mov_ps(FMT == 1 ? 0xFFFF : 0x00FF, sums), cacc[t]);
    }
  }
  for (int t = 0; t < nt; ++t) res[t] = _mm512_reduce_add_ps(_mm512_sub_ps(facc[t], cacc[t]));
}

SWARM_VNNI void matmul_vnni(const uint8_t* w, int type, int rows, int K, const Acts& acts, int T,
                            float* out) {
  // the activation sums the offset corrections are dotted with
  std::vector<float> dxs((size_t)T * (K / 32)), dxs16((size_t)T * (K / 16));
  for (int t = 0; t < T; ++t) {
    const float* dx = acts.dx + (size_t)t * (K / 32);
    const int32_t* sx = acts.sx + (size_t)t * (K / 32);
    const int8_t* q = acts.q + (size_t)t * K;
    for (int j = 0; j < K / 32; ++j) dxs[(size_t)t * (K / 32) + j] = dx[j] * (float)sx[j];
    for (int j = 0; j < K / 16; ++j) {
      int32_t s16 = 0;
      for (int i = 0; i < 16; ++i) s16 += q[16 * j + i];
      dxs16[(size_t)t * (K / 16) + j] = dx[j / 2] * (float)s16;
    }
  }
  const ActsX ax{acts.q, acts.dx, dxs.data(), dxs16.data(), K};
  const size_t row_bytes = row_bytes_of(type, K);
  const int nsb = K / 256;
  auto* fn = type == kGgmlQ4_K     ? row_vnni<0>
             : type == kGgmlQ6_K   ? row_vnni<1>
             : type == kGgmlQ8_0   ? row_vnni<2>
             : type == kGgmlQ4_0   ? row_vnni<3>
             : type == kGgmlIQ4_NL ? row_vnni<4>
             : type == kGgmlMXFP4  ? row_vnni<5>
                                   : row_vnni<6>;
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; ++r) {
    const uint8_t* wr = w + (size_t)r * row_bytes;
    for (int t0 = 0; t0 < T; t0 += kTT) {
      const int nt = T - t0 < kTT ? T - t0 : kTT;
      float res[kTT];
      fn(wr, nsb, ax, t0, nt, res);
      for (int t = 0; t < nt; ++t) out[(size_t)(t0 + t) * rows + r] = res[t];
    }
  }
}

bool use_vnni() {
  static const bool ok = [] {
    const char* e = std::getenv("SWARMLLM_CPU_ISA");
    if (e && std::strcmp(e, "generic") == 0) return false;
    __builtin_cpu_init();
    return __builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bw") &&
           __builtin_cpu_supports("avx512dq") && __builtin_cpu_supports("avx512vl") &&
           __builtin_cpu_supports("avx512vnni");
  }();
  return ok;
}

}  // namespace

const char* cpu_qmatmul_isa() { return use_vnni() ? "avx512vnni" : "generic"; }

int cpu_qmatmul(const uint8_t* w, int type, int rows, int K, const float* x, int T,
                float* out) {
  const bool small_blocks = type == kGgmlQ8_0 || type == kGgmlQ4_0 || type == kGgmlIQ4_NL ||
                            type == kGgmlMXFP4;
  if (K % 256 != 0 && !(small_blocks && K % 32 == 0)) return -1;
  if (type != kGgmlQ4_K && type != kGgmlQ6_K && type != kGgmlIQ4_XS && !small_blocks) return -2;
  std::vector<int8_t> xq((size_t)T * K);
  std::vector<float> dx((size_t)T * (K / 32));
  std::vector<int32_t> sx((size_t)T * (K / 32));
  for (int t = 0; t < T; ++t)
    quantize_row(x + (size_t)t * K, K, xq.data() + (size_t)t * K, dx.data() + (size_t)t * (K / 32),
                 sx.data() + (size_t)t * (K / 32));
  const Acts acts{xq.data(), dx.data(), sx.data(), K};
  if (K % 256 == 0 && use_vnni()) {
    matmul_vnni(w, type, rows, K, acts, T, out);
    return 0;
  }
  const size_t row_bytes = row_bytes_of(type, K);
  const int bvals = small_blocks ? 32 : 256;
  const int nblk = K / bvals;
  const size_t blk_bytes = row_bytes / nblk;
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; ++r) {
    const uint8_t* wr = w + (size_t)r * row_bytes;
    for (int t0 = 0; t0 < T; t0 += kTT) {
      const int nt = T - t0 < kTT ? T - t0 : kTT;
      float acc[kTT] = {};
      for (int b = 0; b < nblk; ++b)
        block_generic(type, wr + (size_t)b * blk_bytes, b * bvals, acts, t0, nt, acc);
      for (int t = 0; t < nt; ++t) out[(size_t)(t0 + t) * rows + r] = acc[t];
    }
  }
  return 0;
}

int cpu_dequant(const uint8_t* w, int type, int rows, int K, float* out) {
  const bool small_blocks = type == kGgmlQ8_0 || type == kGgmlQ4_0 || type == kGgmlIQ4_NL ||
                            type == kGgmlMXFP4;
  if (K % (small_blocks ? 32 : 256) != 0) return -1;
  if (type != kGgmlQ4_K && type != kGgmlQ6_K && type != kGgmlIQ4_XS && !small_blocks) return -2;
  const size_t row_bytes = row_bytes_of(type, K);
  const int bvals = small_blocks ? 32 : 256, nblk = K / bvals;
  const size_t blk_bytes = row_bytes / nblk;
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; ++r) {
    Decoded o;
    for (int b = 0; b < nblk; ++b) {
      decode_block(type, w + (size_t)r * row_bytes + (size_t)b * blk_bytes, o);
      float* dst = out + (size_t)r * K + (size_t)b * bvals;
      for (int i = 0; i < o.n; ++i) dst[i] = o.scale[i / o.sub] * (float)o.q[i] + o.offset[i / o.sub];
    }
  }
  return 0;
}

}  // namespace swarm_native
