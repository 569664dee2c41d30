// GGML/GGUF quantized block formats, device side.
//
// The byte layouts are fixed by the GGUF file format (they must match what
// llama.cpp / gguf-py write, so files interoperate):
//   Q4_0   : {f16 d; u8 qs[16]}                      32 values, 18 B
//   Q8_0   : {f16 d; i8 qs[32]}                      32 values, 34 B
//   Q4_K   : {f16 d; f16 dmin; u8 scales[12]; u8 qs[128]}   256 values, 144 B
//   Q6_K   : {u8 ql[128]; u8 qh[64]; i8 scales[16]; f16 d} 256 values, 210 B
//   IQ4_NL : {f16 d; u8 qs[16]}  non-linear 16-entry codebook, 32 values, 18 B
//   IQ4_XS : {f16 d; u16 scales_h; u8 scales_l[4]; u8 qs[128]} 256 values, 136 B
//   MXFP4  : {u8 e8m0; u8 qs[16]}  OCP MX E2M1 values, 32 values, 17 B
// The reference reads the same blocks through candle's k_quants
// (vendor/candle/candle-core/src/quantized/k_quants.rs) and its CUDA
// dequantizers (vendor/candle/candle-kernels/src/quantized.cu); the code here
// is written from the format definitions, not from those files.
#pragma once
#include "common.cuh"

namespace swarm {

enum GgmlType : int {
  GGML_F32 = 0, GGML_F16 = 1, GGML_Q4_0 = 2, GGML_Q8_0 = 8,
  GGML_Q4_K = 12, GGML_Q6_K = 14, GGML_IQ4_NL = 20, GGML_IQ4_XS = 23,
  GGML_BF16 = 30, GGML_MXFP4 = 39,
};

SW_HOST_DEVICE int ggml_block_values(int t) {
  switch (t) {
    case GGML_Q4_0: case GGML_Q8_0: case GGML_IQ4_NL: case GGML_MXFP4: return 32;
    case GGML_Q4_K: case GGML_Q6_K: case GGML_IQ4_XS: return 256;
    default: return 1;
  }
}
SW_HOST_DEVICE int ggml_block_bytes(int t) {
  switch (t) {
    case GGML_F32: return 4;
    case GGML_F16: case GGML_BF16: return 2;
    case GGML_Q4_0: return 18;
    case GGML_Q8_0: return 34;
    case GGML_Q4_K: return 144;
    case GGML_Q6_K: return 210;
    case GGML_IQ4_NL: return 18;
    case GGML_IQ4_XS: return 136;
    case GGML_MXFP4: return 17;
    default: return 0;
  }
}

// IQ4 codebook (part of the IQ4_NL / IQ4_XS format definition).
__device__ __constant__ static const int8_t kIq4Values[16] = {
    -127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};
// E2M1 magnitudes times two (0, .5, 1, 1.5, 2, 3, 4, 6 -> 0..12); sign in bit 3.
__device__ __constant__ static const int8_t kMxfp4Values[16] = {
    0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};

SW_DEVICE uint16_t ld_u16(const uint8_t* p) { return (uint16_t)p[0] | ((uint16_t)p[1] << 8); }

// Q4_K 6-bit (scale, min) pair for sub-block j (0..7) from the 12-byte field.
SW_DEVICE void q4k_scale_min(int j, const uint8_t* s, int& sc, int& m) {
  if (j < 4) {
    sc = s[j] & 63;
    m = s[j + 4] & 63;
  } else {
    sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
    m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
  }
}

// E8M0 exponent -> float 2^(e-127); the MXFP4 table above is doubled, so the
// block scale used with it is 2^(e-128).
SW_DEVICE float e8m0_half(uint8_t e) {
  // 2^(e-128) built directly from the exponent field; e<2 gives a denormal.
  if (e < 2) return __uint_as_float(0x00200000u << e);
  return __uint_as_float(((uint32_t)(e - 1)) << 23);
}

// Dequantize value `i` (0 <= i < block_values) of one block.
SW_DEVICE float dequant_one(int type, const uint8_t* b, int i) {
  switch (type) {
    case GGML_F32: return *reinterpret_cast<const float*>(b);
    case GGML_F16: return half_bits_to_f(ld_u16(b));
    case GGML_BF16: return __uint_as_float(((uint32_t)ld_u16(b)) << 16);
    case GGML_Q4_0: {
      float d = half_bits_to_f(ld_u16(b));
      int q = (i < 16) ? (b[2 + i] & 0xF) : (b[2 + i - 16] >> 4);
      return d * (float)(q - 8);
    }
    case GGML_Q8_0: {
      float d = half_bits_to_f(ld_u16(b));
      return d * (float)((int8_t)b[2 + i]);
    }
    case GGML_IQ4_NL: {
      float d = half_bits_to_f(ld_u16(b));
      int q = (i < 16) ? (b[2 + i] & 0xF) : (b[2 + i - 16] >> 4);
      return d * (float)kIq4Values[q];
    }
    case GGML_MXFP4: {
      float d = e8m0_half(b[0]);
      int q = (i < 16) ? (b[1 + i] & 0xF) : (b[1 + i - 16] >> 4);
      return d * (float)kMxfp4Values[q];
    }
    case GGML_Q4_K: {
      float d = half_bits_to_f(ld_u16(b)), dmin = half_bits_to_f(ld_u16(b + 2));
      const uint8_t* sc = b + 4;
      const uint8_t* qs = b + 16;
      int g = i >> 6, r = i & 63;        // 64-value group, position inside
      int sub = 2 * g + (r >> 5);        // 32-value sub-block
      int s, m;
      q4k_scale_min(sub, sc, s, m);
      uint8_t byte = qs[32 * g + (r & 31)];
      int q = (r < 32) ? (byte & 0xF) : (byte >> 4);
      return d * s * q - dmin * m;
    }
    case GGML_Q6_K: {
      const uint8_t* ql = b;
      const uint8_t* qh = b + 128;
      const int8_t* sc = reinterpret_cast<const int8_t*>(b + 192);
      float d = half_bits_to_f(ld_u16(b + 208));
      int n = i >> 7, r = i & 127;       // 128-value half
      int quad = r >> 5, l = r & 31;     // which of 4 interleaved 32-runs
      const uint8_t* qlh = ql + 64 * n;
      const uint8_t* qhh = qh + 32 * n;
      int lo = (quad & 1) ? qlh[l + 32] : qlh[l];
      lo = (quad >= 2) ? (lo >> 4) : (lo & 0xF);
      int hi = (qhh[l] >> (2 * quad)) & 3;
      int q = (lo | (hi << 4)) - 32;
      int is = 8 * n + (l >> 4) + 2 * quad;
      return d * sc[is] * q;
    }
    case GGML_IQ4_XS: {
      float d = half_bits_to_f(ld_u16(b));
      uint16_t sh = ld_u16(b + 2);
      const uint8_t* sl = b + 4;
      const uint8_t* qs = b + 8;
      int ib = i >> 5, r = i & 31;
      int ls = ((sl[ib >> 1] >> (4 * (ib & 1))) & 0xF) | (((sh >> (2 * ib)) & 3) << 4);
      float dl = d * (float)(ls - 32);
      uint8_t byte = qs[16 * ib + (r & 15)];
      int q = (r < 16) ? (byte & 0xF) : (byte >> 4);
      return dl * (float)kIq4Values[q];
    }
    default: return 0.f;
  }
}

}  // namespace swarm
