// Embedding gather, RMSNorm and the GEMM epilogues that fuse the small ops of
// a decoder layer into the kernel that reads the GEMM result:
//
//   embed_gather          token ids -> fp32 residual rows (any GGML table type)
//   rmsnorm               fp32 residual -> bf16 normed (GEMM input)
//   epi_residual_rmsnorm  residual += GEMM out; normed = RMSNorm(residual) * w
//                         (replaces the reference's add_rmsnorm_f32,
//                          kernels/fused_decode.cu:119, plus the o/down-proj add)
//   epi_rope_kv           q,k,v from the QKV GEMM: bias, RoPE (GGML "norm"
//                         interleaved pairs or NEOX halves, partial rotary), q ->
//                         bf16, k,v -> fp16 paged cache pages
//                         (replaces heads_first_f32 + rope_partial_f32 +
//                          kv_write_f16: kernels/fused_decode.cu:185,240,
//                          kernels/kv_append.cu:33)
//   epi_swiglu            silu(gate) * up, or gpt-oss clamped SwiGLU
//                         (kernels/fused_decode.cu:47,68)
//   epi_copy              GEMM out -> dense fp32 (logits)
//   mul_f16               x *= y (gated attention: output * sigmoid(gate))
#include "kernels.h"
#include "gemm_out.cuh"
#include "quant_blocks.cuh"

#include <cooperative_groups.h>
namespace cg = cooperative_groups;

namespace swarm {

__global__ void embed_gather_kernel(const uint8_t* __restrict__ table, int type, int hidden,
                                    const int32_t* __restrict__ ids, float* __restrict__ out) {
  pdl_trigger();  // dependents (the next GEMM) may launch and prefetch weights
  pdl_wait();     // what earlier kernels wrote is complete and visible
  const int t = blockIdx.x;
  const int id = ids[t];
  const int bv = ggml_block_values(type), bb = ggml_block_bytes(type);
  const size_t row_bytes = (size_t)(hidden / bv) * bb;
  const uint8_t* row = table + (size_t)id * row_bytes;
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
    const int blk = i / bv;
    out[(size_t)t * hidden + i] = dequant_one(type, row + (size_t)blk * bb, i - blk * bv);
  }
}

template <int kThreads>
__global__ void rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                               __half* __restrict__ out, int dim, float eps) {
  pdl_trigger();  // dependents (the next GEMM) may launch and prefetch weights
  pdl_wait();     // what earlier kernels wrote is complete and visible
  __shared__ float red[32];
  const int t = blockIdx.x;
  const float* xr = x + (size_t)t * dim;
  float ss = 0.f;
  for (int i = threadIdx.x; i < dim; i += kThreads) ss += xr[i] * xr[i];
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / dim + eps);
  for (int i = threadIdx.x; i < dim; i += kThreads)
    out[(size_t)t * dim + i] = __float2half_rn(xr[i] * inv * w[i]);
}

// One CTA per token.  The residual row is staged in shared memory so the
// GEMM partials are read exactly once.
template <int kThreads>
__global__ void epi_residual_rmsnorm_kernel(GemmOut g, float* __restrict__ residual,
                                            const float* __restrict__ bias,
                                            const float* __restrict__ w,
                                            __half* __restrict__ out, float eps,
                                            int out_stride) {
  pdl_trigger();  // dependents (the next GEMM) may launch and prefetch weights
  pdl_wait();     // what earlier kernels wrote is complete and visible
  extern __shared__ float row[];
  __shared__ float red[32];
  const int t = blockIdx.x;
  const int dim = g.rows;
  float* rr = residual + (size_t)t * dim;
  float ss = 0.f;
  const bool vec8 = (dim & 7) == 0 && (reinterpret_cast<uintptr_t>(residual) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(bias) & 15) == 0;
  if (vec8) {
    // eight rows per thread and step: one partial-sum lookup per eight, 16-byte accesses
    for (int i = 8 * threadIdx.x; i < dim; i += 8 * kThreads) {
      float4 g0, g1;
      g.get8(t, i, g0, g1);
      float4 v0 = *reinterpret_cast<const float4*>(rr + i);
      float4 v1 = *reinterpret_cast<const float4*>(rr + i + 4);
      if (bias) {
        const float4 b0 = *reinterpret_cast<const float4*>(bias + i);
        const float4 b1 = *reinterpret_cast<const float4*>(bias + i + 4);
        g0.x += b0.x; g0.y += b0.y; g0.z += b0.z; g0.w += b0.w;
        g1.x += b1.x; g1.y += b1.y; g1.z += b1.z; g1.w += b1.w;
      }
      v0.x += g0.x; v0.y += g0.y; v0.z += g0.z; v0.w += g0.w;
      v1.x += g1.x; v1.y += g1.y; v1.z += g1.z; v1.w += g1.w;
      *reinterpret_cast<float4*>(rr + i) = v0;
      *reinterpret_cast<float4*>(rr + i + 4) = v1;
      *reinterpret_cast<float4*>(row + i) = v0;
      *reinterpret_cast<float4*>(row + i + 4) = v1;
      ss += v0.x * v0.x + v0.y * v0.y + v0.z * v0.z + v0.w * v0.w +
            v1.x * v1.x + v1.y * v1.y + v1.z * v1.z + v1.w * v1.w;
    }
  } else if ((dim & 3) == 0 && (reinterpret_cast<uintptr_t>(residual) & 15) == 0) {
    // four rows per thread and step: 16-byte loads, more bytes in flight
    for (int i = 4 * threadIdx.x; i < dim; i += 4 * kThreads) {
      const float4 gv = g.get4(t, i);
      float4 v = *reinterpret_cast<const float4*>(rr + i);
      v.x += gv.x + (bias ? bias[i] : 0.f);
      v.y += gv.y + (bias ? bias[i + 1] : 0.f);
      v.z += gv.z + (bias ? bias[i + 2] : 0.f);
      v.w += gv.w + (bias ? bias[i + 3] : 0.f);
      *reinterpret_cast<float4*>(rr + i) = v;
      *reinterpret_cast<float4*>(row + i) = v;
      ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
  } else {
    for (int i = threadIdx.x; i < dim; i += kThreads) {
      float v = rr[i] + g.get(t, i) + (bias ? bias[i] : 0.f);
      rr[i] = v;
      row[i] = v;
      ss += v * v;
    }
  }
  if (out == nullptr) return;
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / dim + eps);
  __half* o = out + (size_t)t * out_stride;
  if (vec8 && (out_stride & 7) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(w) & 15) == 0) {
    for (int i = 8 * threadIdx.x; i < dim; i += 8 * kThreads) {
      const float4 a0 = *reinterpret_cast<const float4*>(row + i);
      const float4 a1 = *reinterpret_cast<const float4*>(row + i + 4);
      const float4 w0 = *reinterpret_cast<const float4*>(w + i);
      const float4 w1 = *reinterpret_cast<const float4*>(w + i + 4);
      __align__(16) __half y[8] = {
          __float2half_rn(a0.x * inv * w0.x), __float2half_rn(a0.y * inv * w0.y),
          __float2half_rn(a0.z * inv * w0.z), __float2half_rn(a0.w * inv * w0.w),
          __float2half_rn(a1.x * inv * w1.x), __float2half_rn(a1.y * inv * w1.y),
          __float2half_rn(a1.z * inv * w1.z), __float2half_rn(a1.w * inv * w1.w)};
      *reinterpret_cast<uint4*>(o + i) = *reinterpret_cast<const uint4*>(y);
    }
    return;
  }
  for (int i = threadIdx.x; i < dim; i += kThreads)
    o[i] = __float2half_rn(row[i] * inv * w[i]);
}

// Sandwich-norm variant (Gemma 2/3, GLM-4): the branch output is normalised
// before it joins the residual stream.
//   v = RMSNorm(g + bias) * post_w;  residual += v;  out = RMSNorm(residual) * w
// One CTA per token, the row staged in shared memory.
template <int kThreads>
__global__ void epi_postnorm_residual_rmsnorm_kernel(GemmOut g, float* __restrict__ residual,
                                                     const float* __restrict__ bias,
                                                     const float* __restrict__ post_w,
                                                     const float* __restrict__ w,
                                                     __half* __restrict__ out, float eps,
                                                     int out_stride) {
  pdl_trigger();  // dependents (the next GEMM) may launch and prefetch weights
  pdl_wait();     // what earlier kernels wrote is complete and visible
  extern __shared__ float row[];
  __shared__ float red[32];
  const int t = blockIdx.x;
  const int dim = g.rows;
  float* rr = residual + (size_t)t * dim;
  float ssg = 0.f;
  for (int i = threadIdx.x; i < dim; i += kThreads) {
    const float v = g.get(t, i) + (bias ? bias[i] : 0.f);
    row[i] = v;
    ssg += v * v;
  }
  ssg = block_sum(ssg, red);
  const float invg = rsqrtf(ssg / dim + eps);
  float ss = 0.f;
  for (int i = threadIdx.x; i < dim; i += kThreads) {
    const float v = rr[i] + row[i] * invg * post_w[i];
    rr[i] = v;
    row[i] = v;
    ss += v * v;
  }
  if (out == nullptr) return;
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / dim + eps);
  __half* o = out + (size_t)t * out_stride;
  for (int i = threadIdx.x; i < dim; i += kThreads) o[i] = __float2half_rn(row[i] * inv * w[i]);
}

// Grid (token, group of kRopeHpb heads) over the head list [q | k | v].
// Layout of the QKV GEMM rows: [q heads][k heads][v heads], each head_dim
// wide -- or, for gated attention, each q head as [q | gate].
// Cache layout: [pages][n_kv][page_size][head_dim] fp16.
constexpr int kRopeHpb = 8;

__global__ void epi_rope_kv_kernel(GemmOut g, const float* __restrict__ bias,
                                   const int32_t* __restrict__ positions,
                                   const int32_t* __restrict__ slots,
                                   const float* __restrict__ inv_freq, int n_q, int n_kv,
                                   int head_dim, int rope_dim, int neox, float attn_factor,
                                   __half* __restrict__ q_out, __half* __restrict__ k_cache,
                                   __half* __restrict__ v_cache, int page_size,
                                   const float* __restrict__ q_norm_w,
                                   const float* __restrict__ k_norm_w, float norm_eps,
                                   __half* __restrict__ gate_out) {
  pdl_trigger();  // dependents (the next GEMM) may launch and prefetch weights
  pdl_wait();     // what earlier kernels wrote is complete and visible
  extern __shared__ float sh[];  // kRopeHpb * head_dim floats
  const int t = blockIdx.x;
  const int h0 = blockIdx.y * kRopeHpb;
  const int n_heads = n_q + 2 * n_kv;
  const int nh = min(kRopeHpb, n_heads - h0);
  const int pos = positions[t];
  const int slot = slots ? slots[t] : -1;
  const int page = slot >= 0 ? slot / page_size : 0, off = slot >= 0 ? slot - page * page_size : 0;
  const int q_rows = n_q * head_dim;
  const bool gated = gate_out != nullptr;
  // Stage this CTA's q/k heads (pre-RoPE) in shared memory; v goes straight to
  // the cache.  Four consecutive dims per step (16-byte partial reads); head_dim
  // and the row offsets are multiples of 4.
  for (int i = 4 * threadIdx.x; i < nh * head_dim; i += 4 * blockDim.x) {
    const int j = i / head_dim, d = i - j * head_dim;
    const int hh = h0 + j;
    const int lr = hh * head_dim + d;  // logical row
    const int gr = gated ? (hh < n_q ? lr + hh * head_dim : lr + q_rows) : lr;
    float4 v = g.get4(t, gr);
    if (bias) {
      v.x += bias[lr];
      v.y += bias[lr + 1];
      v.z += bias[lr + 2];
      v.w += bias[lr + 3];
    }
    if (hh < n_q + n_kv) {
      *reinterpret_cast<float4*>(sh + i) = v;
      if (gated && hh < n_q) {
        const float4 gv = g.get4(t, gr + head_dim);
        __half* go = gate_out + (size_t)t * q_rows + lr;
        go[0] = __float2half_rn(1.f / (1.f + __expf(-gv.x)));
        go[1] = __float2half_rn(1.f / (1.f + __expf(-gv.y)));
        go[2] = __float2half_rn(1.f / (1.f + __expf(-gv.z)));
        go[3] = __float2half_rn(1.f / (1.f + __expf(-gv.w)));
      }
    } else if (slot >= 0) {
      const int hv = hh - n_q - n_kv;
      __align__(8) __half h4[4] = {__float2half_rn(v.x), __float2half_rn(v.y),
                                   __float2half_rn(v.z), __float2half_rn(v.w)};
      *reinterpret_cast<uint2*>(v_cache + (((size_t)page * n_kv + hv) * page_size + off) * head_dim +
                                d) = *reinterpret_cast<const uint2*>(h4);
    }
  }
  __syncthreads();
  // Optional per-head RMSNorm of q and k (Qwen3-style qk-norm); one warp per head.
  if (q_norm_w != nullptr) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int j = warp; j < nh; j += nw) {
      const int hh = h0 + j;
      if (hh >= n_q + n_kv) continue;
      float* x = sh + j * head_dim;
      float ss = 0.f;
      for (int d = lane; d < head_dim; d += 32) ss += x[d] * x[d];
      ss = warp_sum(ss);
      const float inv = rsqrtf(ss / head_dim + norm_eps);
      const float* wn = (hh < n_q) ? q_norm_w : k_norm_w;
      for (int d = lane; d < head_dim; d += 32) x[d] = x[d] * inv * wn[d];
    }
    __syncthreads();
  }
  const int half = rope_dim / 2, hd2 = head_dim / 2;
  if ((half & 1) == 0 && (rope_dim & 3) == 0 && (head_dim & 3) == 0 &&
      ((reinterpret_cast<uintptr_t>(q_out) | reinterpret_cast<uintptr_t>(k_cache)) & 7) == 0) {
    // Two adjacent dimension pairs per thread (pair index p even): the rotated
    // halves go out as 4-byte stores (NEOX: p, p + 1 and p + half, p + half + 1)
    // or one 8-byte store (interleaved pairs, and the unrotated tail).
    const int hq = hd2 >> 1;
    for (int i = threadIdx.x; i < nh * hq; i += blockDim.x) {
      const int j = i / hq, p = 2 * (i - j * hq);
      const int hh = h0 + j;
      if (hh >= n_q + n_kv) continue;
      __half* dst;
      if (hh < n_q) {
        dst = q_out + ((size_t)t * n_q + hh) * head_dim;
      } else if (slot >= 0) {
        dst = k_cache + (((size_t)page * n_kv + (hh - n_q)) * page_size + off) * head_dim;
      } else {
        continue;
      }
      const float* x = sh + j * head_dim;
      if (p < half) {   // both pairs rotated (half is even)
        float s0, c0, s1, c1;
        sincosf((float)pos * inv_freq[p], &s0, &c0);
        sincosf((float)pos * inv_freq[p + 1], &s1, &c1);
        c0 *= attn_factor; s0 *= attn_factor; c1 *= attn_factor; s1 *= attn_factor;
        if (neox) {
          const float a0 = x[p], a1 = x[p + 1], b0 = x[p + half], b1 = x[p + 1 + half];
          *reinterpret_cast<__half2*>(dst + p) =
              __floats2half2_rn(a0 * c0 - b0 * s0, a1 * c1 - b1 * s1);
          *reinterpret_cast<__half2*>(dst + p + half) =
              __floats2half2_rn(b0 * c0 + a0 * s0, b1 * c1 + a1 * s1);
        } else {
          const float a0 = x[2 * p], b0 = x[2 * p + 1], a1 = x[2 * p + 2], b1 = x[2 * p + 3];
          __align__(8) __half2 y[2] = {__floats2half2_rn(a0 * c0 - b0 * s0, b0 * c0 + a0 * s0),
                                       __floats2half2_rn(a1 * c1 - b1 * s1, b1 * c1 + a1 * s1)};
          *reinterpret_cast<uint2*>(dst + 2 * p) = *reinterpret_cast<const uint2*>(y);
        }
      } else {          // both pairs in the unrotated tail: four contiguous values
        const int d0 = rope_dim + 2 * (p - half);
        __align__(8) __half2 y[2] = {__floats2half2_rn(x[d0], x[d0 + 1]),
                                     __floats2half2_rn(x[d0 + 2], x[d0 + 3])};
        *reinterpret_cast<uint2*>(dst + d0) = *reinterpret_cast<const uint2*>(y);
      }
    }
    return;
  }
  // One thread per dimension pair: rotated pairs share one sincos; the
  // unrotated tail (partial RoPE) is copied pairwise.
  for (int i = threadIdx.x; i < nh * hd2; i += blockDim.x) {
    const int j = i / hd2, p = i - j * hd2;
    const int hh = h0 + j;
    if (hh >= n_q + n_kv) continue;
    const float* x = sh + j * head_dim;
    int d0, d1;
    float y0, y1;
    if (p < half) {
      if (neox) {
        d0 = p;
        d1 = p + half;
      } else {
        d0 = 2 * p;
        d1 = 2 * p + 1;
      }
      float sn, cs;
      sincosf((float)pos * inv_freq[p], &sn, &cs);
      cs *= attn_factor;
      sn *= attn_factor;
      y0 = x[d0] * cs - x[d1] * sn;
      y1 = x[d1] * cs + x[d0] * sn;
    } else {
      d0 = rope_dim + 2 * (p - half);
      d1 = d0 + 1;
      y0 = x[d0];
      y1 = x[d1];
    }
    __half* dst;
    if (hh < n_q) {
      dst = q_out + ((size_t)t * n_q + hh) * head_dim;
    } else if (slot >= 0) {
      const int hk = hh - n_q;
      dst = k_cache + (((size_t)page * n_kv + hk) * page_size + off) * head_dim;
    } else {
      continue;
    }
    dst[d0] = __float2half_rn(y0);
    dst[d1] = __float2half_rn(y1);
  }
}

// GELU with the tanh approximation (Hendrycks & Gimpel 2016): the Gemma FFN.
SW_DEVICE float gelu_tanh(float x) {
  const float k0 = 0.7978845608028654f;  // sqrt(2 / pi)
  return 0.5f * x * (1.f + tanhf(k0 * (x + 0.044715f * x * x * x)));
}

// rows [0, F) are gate, [F, 2F) are up (or interleaved for gpt-oss: even=gate,
// odd=up when `interleaved`).  kind 0: silu(g)*u.  kind 1: gpt-oss clamped
// SwiGLU x=min(g,limit), u=clamp(u,-limit,limit), x*sigmoid(alpha*x)*(u+1).
// kind 2: gelu_tanh(g)*u (GeGLU).
__global__ void epi_swiglu_kernel(GemmOut g, const float* __restrict__ bias, int F, int kind,
                                  int interleaved, float alpha, float limit,
                                  __half* __restrict__ out) {
  pdl_trigger();  // dependents (the next GEMM) may launch and prefetch weights
  pdl_wait();     // what earlier kernels wrote is complete and visible
  const int t = blockIdx.y;
  if (!interleaved && (F & 7) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0) {
    // eight features per thread and step: one partial-sum lookup per eight, 16-byte stores
    for (int i = 8 * (blockIdx.x * blockDim.x + threadIdx.x); i < F; i += 8 * gridDim.x * blockDim.x) {
      float4 g0, g1, u0, u1;
      g.get8(t, i, g0, g1);
      g.get8(t, F + i, u0, u1);
      const float gs[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
      const float us[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
      __align__(16) __half y[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float gv = gs[e] + (bias ? bias[i + e] : 0.f);
        float uv = us[e] + (bias ? bias[F + i + e] : 0.f);
        if (kind == 0) {
          y[e] = __float2half_rn(__fdividef(gv, 1.f + __expf(-gv)) * uv);
        } else if (kind == 2) {
          y[e] = __float2half_rn(gelu_tanh(gv) * uv);
        } else {
          gv = fminf(gv, limit);
          uv = fminf(fmaxf(uv, -limit), limit);
          y[e] = __float2half_rn(__fdividef(gv, 1.f + __expf(-alpha * gv)) * (uv + 1.f));
        }
      }
      *reinterpret_cast<uint4*>(out + (size_t)t * F + i) = *reinterpret_cast<const uint4*>(y);
    }
    return;
  }
  if (!interleaved && (F & 3) == 0 && (reinterpret_cast<uintptr_t>(out) & 7) == 0) {
    // four features per thread and step, 16-byte loads
    for (int i = 4 * (blockIdx.x * blockDim.x + threadIdx.x); i < F; i += 4 * gridDim.x * blockDim.x) {
      const float4 g4 = g.get4(t, i), u4 = g.get4(t, F + i);
      const float gs[4] = {g4.x, g4.y, g4.z, g4.w}, us[4] = {u4.x, u4.y, u4.z, u4.w};
      __align__(8) __half y[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float gv = gs[e] + (bias ? bias[i + e] : 0.f);
        float uv = us[e] + (bias ? bias[F + i + e] : 0.f);
        if (kind == 0) {
          y[e] = __float2half_rn(silu(gv) * uv);
        } else if (kind == 2) {
          y[e] = __float2half_rn(gelu_tanh(gv) * uv);
        } else {
          gv = fminf(gv, limit);
          uv = fminf(fmaxf(uv, -limit), limit);
          y[e] = __float2half_rn(gv / (1.f + __expf(-alpha * gv)) * (uv + 1.f));
        }
      }
      *reinterpret_cast<uint2*>(out + (size_t)t * F + i) = *reinterpret_cast<const uint2*>(y);
    }
    return;
  }
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < F; i += gridDim.x * blockDim.x) {
    const int rg = interleaved ? 2 * i : i;
    const int ru = interleaved ? 2 * i + 1 : F + i;
    float gv = g.get(t, rg) + (bias ? bias[rg] : 0.f);
    float uv = g.get(t, ru) + (bias ? bias[ru] : 0.f);
    float y;
    if (kind == 0) {
      y = silu(gv) * uv;
    } else if (kind == 2) {
      y = gelu_tanh(gv) * uv;
    } else {
      gv = fminf(gv, limit);
      uv = fminf(fmaxf(uv, -limit), limit);
      y = gv / (1.f + __expf(-alpha * gv)) * (uv + 1.f);
    }
    out[(size_t)t * F + i] = __float2half_rn(y);
  }
}

__global__ void epi_copy_kernel(GemmOut g, const float* __restrict__ bias, float* __restrict__ out,
                                int out_stride) {
  pdl_trigger();  // dependents (the next GEMM) may launch and prefetch weights
  pdl_wait();     // what earlier kernels wrote is complete and visible
  const int t = blockIdx.y;
  if ((g.rows & 3) == 0 && (out_stride & 3) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0) {
    for (int i = 4 * (blockIdx.x * blockDim.x + threadIdx.x); i < g.rows;
         i += 4 * gridDim.x * blockDim.x) {
      float4 v = g.get4(t, i);
      if (bias) {
        v.x += bias[i];
        v.y += bias[i + 1];
        v.z += bias[i + 2];
        v.w += bias[i + 3];
      }
      *reinterpret_cast<float4*>(out + (size_t)t * out_stride + i) = v;
    }
    return;
  }
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < g.rows; i += gridDim.x * blockDim.x)
    out[(size_t)t * out_stride + i] = g.get(t, i) + (bias ? bias[i] : 0.f);
}

__global__ void mul_f16_kernel(__half* __restrict__ x, const __half* __restrict__ y, size_t n) {
  pdl_trigger();  // dependents (the next GEMM) may launch and prefetch weights
  pdl_wait();     // what earlier kernels wrote is complete and visible
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    x[i] = __hmul(x[i], y[i]);
}

__global__ void f32_to_f16_kernel(const float* __restrict__ x, __half* __restrict__ y,
                                   size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    y[i] = __float2half_rn(x[i]);
}

}  // namespace swarm

using namespace swarm;

void launch_embed_gather(const void* table, int type, int hidden, const int32_t* ids, int n,
                         float* out, cudaStream_t s) {
  if (n <= 0) return;
  launch_pdl(embed_gather_kernel, dim3(n), dim3(256), 0, s, (const uint8_t*)table, type, hidden,
             ids, out);
  SW_LAUNCH_CHECK();
}

void launch_rmsnorm(const float* x, const float* w, __half* out, int rows, int dim,
                    float eps, cudaStream_t s) {
  if (rows <= 0) return;
  launch_pdl(rmsnorm_kernel<512>, dim3(rows), dim3(512), 0, s, x, w, out, dim, eps);
  SW_LAUNCH_CHECK();
}

// Small batches: one thread-block cluster of kClusterNorm CTAs per token, each
// CTA owning a contiguous slice of the row; the row's sum of squares is
// reduced through distributed shared memory (every CTA reads the others'
// partials), so a decode step's few tokens still spread over many SMs.
constexpr int kClusterNorm = 8;

__global__ void __launch_bounds__(256) epi_residual_rmsnorm_cluster_kernel(
    GemmOut g, float* __restrict__ residual, const float* __restrict__ bias,
    const float* __restrict__ w, __half* __restrict__ out, float eps, int out_stride) {
  pdl_trigger();  // dependents (the next GEMM) may launch and prefetch weights
  pdl_wait();     // what earlier kernels wrote is complete and visible
  cg::cluster_group cluster = cg::this_cluster();
  __shared__ float part;
  __shared__ float red[32];
  extern __shared__ float slice[];
  const int cr = (int)cluster.block_rank(), cn = (int)cluster.num_blocks();
  const int t = blockIdx.x / cn;
  const int dim = g.rows;
  const int per = (dim + cn - 1) / cn;
  const int lo = cr * per, hi = min(dim, lo + per);
  float* rr = residual + (size_t)t * dim;
  float ss = 0.f;
  for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    const float v = rr[i] + g.get(t, i) + (bias ? bias[i] : 0.f);
    rr[i] = v;
    slice[i - lo] = v;
    ss += v * v;
  }
  ss = block_sum(ss, red);
  if (threadIdx.x == 0) part = ss;
  cluster.sync();
  float tot = 0.f;
  for (int r = 0; r < cn; ++r) tot += *cluster.map_shared_rank(&part, r);
  cluster.sync();  // peers finished reading `part` before any CTA exits
  if (out == nullptr) return;
  const float inv = rsqrtf(tot / dim + eps);
  for (int i = lo + threadIdx.x; i < hi; i += blockDim.x)
    out[(size_t)t * out_stride + i] = __float2half_rn(slice[i - lo] * inv * w[i]);
}

void launch_epi_residual_rmsnorm(const GemmOut& g, float* residual, const float* bias,
                                 const float* w, __half* out, float eps, int out_stride,
                                 cudaStream_t s, const float* post_w) {
  if (g.T <= 0) return;
  if (post_w != nullptr) {
    const size_t sm = (size_t)g.rows * sizeof(float);
    if (sm > 48 * 1024)
      cudaFuncSetAttribute(epi_postnorm_residual_rmsnorm_kernel<512>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    launch_pdl(epi_postnorm_residual_rmsnorm_kernel<512>, dim3(g.T), dim3(512), sm, s, g,
               residual, bias, post_w, w, out, eps, out_stride ? out_stride : g.rows);
    SW_LAUNCH_CHECK();
    return;
  }
  if (g.T < 64) {
    const int per = (g.rows + kClusterNorm - 1) / kClusterNorm;
    launch_pdl_cluster(epi_residual_rmsnorm_cluster_kernel, dim3(g.T * kClusterNorm), dim3(256),
                       (size_t)per * sizeof(float), s, kClusterNorm, g, residual, bias, w, out,
                       eps, out_stride ? out_stride : g.rows);
    SW_LAUNCH_CHECK();
    return;
  }
  size_t sm = (size_t)g.rows * sizeof(float);
  if (sm > 48 * 1024)
    cudaFuncSetAttribute(epi_residual_rmsnorm_kernel<512>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  launch_pdl(epi_residual_rmsnorm_kernel<512>, dim3(g.T), dim3(512), sm, s, g, residual, bias, w,
             out, eps, out_stride ? out_stride : g.rows);
  SW_LAUNCH_CHECK();
}

void launch_epi_rope_kv(const GemmOut& g, const float* bias, const int32_t* positions,
                        const int32_t* slots, const float* inv_freq, int n_q, int n_kv,
                        int head_dim, int rope_dim, int neox, float attn_factor,
                        __half* q_out, __half* k_cache, __half* v_cache, int page_size,
                        const float* q_norm_w, const float* k_norm_w, float norm_eps,
                        __half* gate_out, cudaStream_t s) {
  if (g.T <= 0) return;
  const size_t sm = (size_t)kRopeHpb * head_dim * sizeof(float);
  const int groups = (n_q + 2 * n_kv + kRopeHpb - 1) / kRopeHpb;
  launch_pdl(epi_rope_kv_kernel, dim3(g.T, groups), dim3(256), sm, s, g, bias, positions, slots,
             inv_freq, n_q, n_kv, head_dim, rope_dim, neox, attn_factor, q_out, k_cache, v_cache,
             page_size, q_norm_w, k_norm_w, norm_eps, gate_out);
  SW_LAUNCH_CHECK();
}

void launch_epi_swiglu(const GemmOut& g, const float* bias, int F, int kind, int interleaved,
                       float alpha, float limit, __half* out, cudaStream_t s) {
  if (g.T <= 0) return;
  // one step per thread on the vector paths (8 or 4 features), else one feature
  const int per = (!interleaved && (F & 7) == 0) ? 8 : (!interleaved && (F & 3) == 0) ? 4 : 1;
  const int need = (F + per * 256 - 1) / (per * 256);
  dim3 grid(need < 64 ? need : 64, g.T);
  launch_pdl(epi_swiglu_kernel, grid, dim3(256), 0, s, g, bias, F, kind, interleaved, alpha,
             limit, out);
  SW_LAUNCH_CHECK();
}

void launch_epi_copy(const GemmOut& g, const float* bias, float* out, int out_stride,
                     cudaStream_t s) {
  if (g.T <= 0) return;
  dim3 grid((g.rows + 255) / 256 < 256 ? (g.rows + 255) / 256 : 256, g.T);
  launch_pdl(epi_copy_kernel, grid, dim3(256), 0, s, g, bias, out,
             out_stride ? out_stride : g.rows);
  SW_LAUNCH_CHECK();
}

void launch_f32_to_f16(const float* x, __half* y, size_t n, cudaStream_t s) {
  if (n == 0) return;
  int blocks = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
  f32_to_f16_kernel<<<blocks, 256, 0, s>>>(x, y, n);
  SW_LAUNCH_CHECK();
}

void launch_mul_f16(__half* x, const __half* y, size_t n, cudaStream_t s) {
  if (n == 0) return;
  int blocks = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
  mul_f16_kernel<<<blocks, 256, 0, s>>>(x, y, n);
  SW_LAUNCH_CHECK();
}
