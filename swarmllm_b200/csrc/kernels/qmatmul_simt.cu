// Quantized matmul on CUDA cores, any supported GGML block type, weights in
// the GGUF file's own row-major block layout:  out[t][r] = sum_k W[r][k] x[t][k].
//
// This is the general path (every block type, any K that is a multiple of the
// block size, no repacking) and the on-device oracle for the tensor-core GEMM.
// One warp owns one output row; each lane walks 32-value sub-blocks, dequantizes
// them into registers and multiplies them with up to kMaxT token rows.
// The reference's equivalents are candle's dmmv/mmvq kernels
// (vendor/candle/candle-kernels/src/quantized.cu) dispatched from
// vendor/candle/candle-core/src/quantized/cuda.rs:472,519.
#include "kernels.h"
#include "quant_blocks.cuh"

namespace swarm {

// Dequantize the 32-value sub-block `sub` of one block into v[32].
template <int TYPE>
SW_DEVICE void dequant_sub32(const uint8_t* __restrict__ b, int sub, float v[32]) {
  if constexpr (TYPE == GGML_Q4_0 || TYPE == GGML_IQ4_NL) {
    const float d = half_bits_to_f(ld_u16(b));
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint8_t q = b[2 + j];
      if constexpr (TYPE == GGML_Q4_0) {
        v[j] = d * (float)((q & 0xF) - 8);
        v[j + 16] = d * (float)((q >> 4) - 8);
      } else {
        v[j] = d * (float)kIq4Values[q & 0xF];
        v[j + 16] = d * (float)kIq4Values[q >> 4];
      }
    }
  } else if constexpr (TYPE == GGML_MXFP4) {
    const float d = e8m0_half(b[0]);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint8_t q = b[1 + j];
      v[j] = d * (float)kMxfp4Values[q & 0xF];
      v[j + 16] = d * (float)kMxfp4Values[q >> 4];
    }
  } else if constexpr (TYPE == GGML_Q8_0) {
    const float d = half_bits_to_f(ld_u16(b));
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = d * (float)((int8_t)b[2 + j]);
  } else if constexpr (TYPE == GGML_Q4_K) {
    const float d = half_bits_to_f(ld_u16(b)), dmin = half_bits_to_f(ld_u16(b + 2));
    int sc, m;
    q4k_scale_min(sub, b + 4, sc, m);
    const float d1 = d * sc, m1 = dmin * m;
    const uint8_t* qs = b + 16 + 32 * (sub >> 1);
    const int shift = (sub & 1) * 4;
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = d1 * (float)((qs[j] >> shift) & 0xF) - m1;
  } else if constexpr (TYPE == GGML_Q6_K) {
    const int n = sub >> 2, quad = sub & 3;
    const uint8_t* ql = b + 64 * n + ((quad & 1) ? 32 : 0);
    const uint8_t* qh = b + 128 + 32 * n;
    const int8_t* sc = reinterpret_cast<const int8_t*>(b + 192) + 8 * n + 2 * quad;
    const float d = half_bits_to_f(ld_u16(b + 208));
    const float d0 = d * sc[0], d1 = d * sc[1];
#pragma unroll
    for (int l = 0; l < 32; ++l) {
      int lo = (quad >= 2) ? (ql[l] >> 4) : (ql[l] & 0xF);
      int hi = (qh[l] >> (2 * quad)) & 3;
      v[l] = ((l < 16) ? d0 : d1) * (float)((lo | (hi << 4)) - 32);
    }
  } else if constexpr (TYPE == GGML_IQ4_XS) {
    const float d = half_bits_to_f(ld_u16(b));
    const uint16_t sh = ld_u16(b + 2);
    const int ls = ((b[4 + (sub >> 1)] >> (4 * (sub & 1))) & 0xF) | (((sh >> (2 * sub)) & 3) << 4);
    const float dl = d * (float)(ls - 32);
    const uint8_t* qs = b + 8 + 16 * sub;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      v[j] = dl * (float)kIq4Values[qs[j] & 0xF];
      v[j + 16] = dl * (float)kIq4Values[qs[j] >> 4];
    }
  } else if constexpr (TYPE == GGML_F16) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = half_bits_to_f(ld_u16(b + 2 * (32 * sub + j)));
  } else if constexpr (TYPE == GGML_BF16) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(((uint32_t)ld_u16(b + 2 * (32 * sub + j))) << 16);
  } else if constexpr (TYPE == GGML_F32) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = reinterpret_cast<const float*>(b)[32 * sub + j];
  }
}

template <int TYPE, int kMaxT>
__global__ void __launch_bounds__(256) qmatmul_simt_kernel(
    const uint8_t* __restrict__ w, int rows, int K, const __half* __restrict__ x,
    int x_stride, int T, float* __restrict__ out, int out_stride) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  // Float types are treated as 32-value "blocks" of 32*elem bytes.
  constexpr bool kFloat = (TYPE == GGML_F16 || TYPE == GGML_BF16 || TYPE == GGML_F32);
  const int bv = kFloat ? 32 : ggml_block_values(TYPE);
  const int bb = kFloat ? 32 * ggml_block_bytes(TYPE) : ggml_block_bytes(TYPE);
  const int subs_per_block = bv / 32;
  const size_t row_bytes = (size_t)(K / bv) * bb;
  const uint8_t* wr = w + (size_t)warp * row_bytes;
  float acc[kMaxT];
#pragma unroll
  for (int t = 0; t < kMaxT; ++t) acc[t] = 0.f;
  const int n_sub = K / 32;
  for (int u = lane; u < n_sub; u += 32) {
    const int blk = u / subs_per_block, sub = u - blk * subs_per_block;
    float v[32];
    dequant_sub32<TYPE>(wr + (size_t)blk * bb, kFloat ? 0 : sub, v);
#pragma unroll
    for (int t = 0; t < kMaxT; ++t) {
      if (t < T) {
        const uint4* xp = reinterpret_cast<const uint4*>(x + (size_t)t * x_stride + 32 * u);
        float a = 0.f;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint4 q = __ldg(xp + c);
          const __half2* h = reinterpret_cast<const __half2*>(&q);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float2 f = __half22float2(h[e]);
            a = fmaf(v[8 * c + 2 * e], f.x, a);
            a = fmaf(v[8 * c + 2 * e + 1], f.y, a);
          }
        }
        acc[t] += a;
      }
    }
  }
#pragma unroll
  for (int t = 0; t < kMaxT; ++t) {
    if (t < T) {
      float s = warp_sum(acc[t]);
      if (lane == 0) out[(size_t)t * out_stride + warp] = s;
    }
  }
}

template <int TYPE>
static void dispatch_t(const uint8_t* w, int rows, int K, const __half* x, int x_stride,
                       int T, float* out, int out_stride, cudaStream_t s) {
  const int blocks = (rows * 32 + 255) / 256;
  for (int t0 = 0; t0 < T; t0 += 8) {
    const int tc = (T - t0) < 8 ? (T - t0) : 8;
    const __half* xs = x + (size_t)t0 * x_stride;
    float* os = out + (size_t)t0 * out_stride;
    if (tc <= 1)
      qmatmul_simt_kernel<TYPE, 1><<<blocks, 256, 0, s>>>(w, rows, K, xs, x_stride, tc, os, out_stride);
    else if (tc <= 4)
      qmatmul_simt_kernel<TYPE, 4><<<blocks, 256, 0, s>>>(w, rows, K, xs, x_stride, tc, os, out_stride);
    else
      qmatmul_simt_kernel<TYPE, 8><<<blocks, 256, 0, s>>>(w, rows, K, xs, x_stride, tc, os, out_stride);
  }
}

// GGML blocks -> fp16 [rows][K], two values per thread (the prefill path of
// quantized types without a tensor-core kernel of their own: dequantize once,
// then the dense tcgen05 GEMM).  Memory-bound; the block header re-reads hit L1.
template <int TYPE>
__global__ void dequant_f16_kernel(const uint8_t* __restrict__ w, int rows, int K,
                                   __half* __restrict__ out) {
  const int BV = ggml_block_values(TYPE), BB = ggml_block_bytes(TYPE);
  const size_t n2 = (size_t)rows * K / 2;
  for (size_t p = blockIdx.x * (size_t)blockDim.x + threadIdx.x; p < n2;
       p += (size_t)gridDim.x * blockDim.x) {
    const size_t e = 2 * p;
    const int r = (int)(e / K), k = (int)(e - (size_t)r * K);
    const uint8_t* blk = w + ((size_t)r * (K / BV) + k / BV) * BB;
    const int i = k % BV;
    const float v0 = dequant_one(TYPE, blk, i), v1 = dequant_one(TYPE, blk, i + 1);
    reinterpret_cast<__half2*>(out)[p] = __floats2half2_rn(v0, v1);
  }
}

template <int TYPE>
static void dequant_t(const uint8_t* w, int rows, int K, __half* out, cudaStream_t s) {
  const size_t n2 = (size_t)rows * K / 2;
  const int blocks = (int)((n2 + 255) / 256 < 65536 ? (n2 + 255) / 256 : 65536);
  dequant_f16_kernel<TYPE><<<blocks, 256, 0, s>>>(w, rows, K, out);
}

}  // namespace swarm

using namespace swarm;

int launch_dequant_f16(const void* w, int type, int rows, int K, __half* out, cudaStream_t s) {
  if (rows <= 0 || K <= 0) return 0;
  if (K % 2 != 0 || K % ggml_block_values(type) != 0) return -1;
  const uint8_t* wb = (const uint8_t*)w;
  switch (type) {
    case GGML_Q4_0: dequant_t<GGML_Q4_0>(wb, rows, K, out, s); break;
    case GGML_Q8_0: dequant_t<GGML_Q8_0>(wb, rows, K, out, s); break;
    case GGML_Q4_K: dequant_t<GGML_Q4_K>(wb, rows, K, out, s); break;
    case GGML_Q6_K: dequant_t<GGML_Q6_K>(wb, rows, K, out, s); break;
    case GGML_IQ4_NL: dequant_t<GGML_IQ4_NL>(wb, rows, K, out, s); break;
    case GGML_IQ4_XS: dequant_t<GGML_IQ4_XS>(wb, rows, K, out, s); break;
    case GGML_MXFP4: dequant_t<GGML_MXFP4>(wb, rows, K, out, s); break;
    default: return -2;
  }
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -3;
}

int launch_qmatmul_simt(const void* w, int type, int rows, int K, const __half* x,
                        int x_stride, int T, float* out, int out_stride, cudaStream_t s) {
  if (T <= 0 || rows <= 0) return 0;
  const uint8_t* wb = (const uint8_t*)w;
  switch (type) {
    case GGML_Q4_0: dispatch_t<GGML_Q4_0>(wb, rows, K, x, x_stride, T, out, out_stride, s); break;
    case GGML_Q8_0: dispatch_t<GGML_Q8_0>(wb, rows, K, x, x_stride, T, out, out_stride, s); break;
    case GGML_Q4_K: dispatch_t<GGML_Q4_K>(wb, rows, K, x, x_stride, T, out, out_stride, s); break;
    case GGML_Q6_K: dispatch_t<GGML_Q6_K>(wb, rows, K, x, x_stride, T, out, out_stride, s); break;
    case GGML_IQ4_NL: dispatch_t<GGML_IQ4_NL>(wb, rows, K, x, x_stride, T, out, out_stride, s); break;
    case GGML_IQ4_XS: dispatch_t<GGML_IQ4_XS>(wb, rows, K, x, x_stride, T, out, out_stride, s); break;
    case GGML_MXFP4: dispatch_t<GGML_MXFP4>(wb, rows, K, x, x_stride, T, out, out_stride, s); break;
    case GGML_F16: dispatch_t<GGML_F16>(wb, rows, K, x, x_stride, T, out, out_stride, s); break;
    case GGML_BF16: dispatch_t<GGML_BF16>(wb, rows, K, x, x_stride, T, out, out_stride, s); break;
    case GGML_F32: dispatch_t<GGML_F32>(wb, rows, K, x, x_stride, T, out, out_stride, s); break;
    default: return -1;
  }
  SW_LAUNCH_CHECK();
  return 0;
}
