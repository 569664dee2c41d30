// Gated DeltaNet (linear attention of the Qwen3-Next-style hybrid) on sm_100a.
//
//   ssm_conv_silu   causal depthwise conv1d (kernel 4) over the q|k|v channels
//                   of the in-projection, with per-sequence carried state, then
//                   SiLU.  Rows of one sequence are consecutive in the batch.
//   delta_rule      the gated delta rule per (sequence, value head), state
//                   S[dk][dv] in fp32:
//                     S <- S * exp(g_t)
//                     d  = (v_t - S^T k_t) * beta_t
//                     S <- S + k_t d^T
//                     o_t = S^T q_t
//                   with q, k L2-normalised (q also scaled by dk^-1/2),
//                   beta = sigmoid(b), g = A * softplus(a + dt_bias), then the
//                   gated RMSNorm of the head output, rmsnorm(o) * w * silu(z),
//                   written as fp16 input of the out-projection GEMM.
//   delta_chunk     the same recurrence for prefill, evaluated a chunk of
//                   tokens at a time (see deltanet_chunk.cu).
//
// Sequence table (int32 [S][4]): row0, nrows, state slot, position of row0.
// A sequence whose row0 sits at position 0 starts from a zero state.
//
// Reference: kernels/delta_rule.cu:212-246 (delta_rule_f32_d*), :324
// (ssm_conv_silu_f32_k4), :421 (ssm_gates_f32), :544 (l2_norm_rows_f32).
#include "kernels.h"
#include "gemm_out.cuh"
#include "common.cuh"

namespace swarm {

template <int K>
__global__ void ssm_conv_silu_kernel(GemmOut g, const float* __restrict__ w, int C,
                                     float* __restrict__ state, const int4* __restrict__ seqs,
                                     float* __restrict__ out) {
  const int s = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const int4 sq = seqs[s];
  const int r0 = sq.x, n = sq.y, slot = sq.z, p0 = sq.w;
  if (n <= 0) return;
  float win[K - 1], wk[K];
#pragma unroll
  for (int i = 0; i < K; ++i) wk[i] = w[(size_t)c * K + i];
  float* st = state + (size_t)slot * (K - 1) * C;
#pragma unroll
  for (int i = 0; i < K - 1; ++i) win[i] = p0 == 0 ? 0.f : st[(size_t)i * C + c];
  for (int t = 0; t < n; ++t) {
    const float v = g.get(r0 + t, c);
    float acc = wk[K - 1] * v;
#pragma unroll
    for (int i = 0; i < K - 1; ++i) acc += wk[i] * win[i];
#pragma unroll
    for (int i = 0; i < K - 2; ++i) win[i] = win[i + 1];
    win[K - 2] = v;
    out[(size_t)(r0 + t) * C + c] = silu(acc);
  }
#pragma unroll
  for (int i = 0; i < K - 1; ++i) st[(size_t)i * C + c] = win[i];
}

// Block-wide sums of two values for a 128-thread block (4 warps).
SW_DEVICE float2 block_sum2_128(float a, float b, float* red) {
  a = warp_sum(a);
  b = warp_sum(b);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { red[warp] = a; red[4 + warp] = b; }
  __syncthreads();
  const float2 r = make_float2(red[0] + red[1] + red[2] + red[3], red[4] + red[5] + red[6] + red[7]);
  __syncthreads();
  return r;
}

// One CTA (D threads) per (sequence, value head); thread j owns column j of S.
template <int D>
__global__ void __launch_bounds__(D) delta_rule_kernel(
    const float* __restrict__ qkv, int C, int nk, int nv, GemmOut gba,
    const float* __restrict__ dt_bias, const float* __restrict__ A, GemmOut gz,
    const float* __restrict__ norm_w, float eps, float* __restrict__ state,
    const int4* __restrict__ seqs, __half* __restrict__ out) {
  static_assert(D == 128, "one thread per value channel, 4 warps");
  __shared__ float qs[D], ks[D], red[8];
  const int s = blockIdx.x, h = blockIdx.y, j = threadIdx.x;
  const int4 sq = seqs[s];
  const int r0 = sq.x, n = sq.y, slot = sq.z, p0 = sq.w;
  if (n <= 0) return;
  const int kh = h / (nv / nk);
  const float scale = rsqrtf((float)D);
  float S[D];
  float* st = state + ((size_t)slot * nv + h) * D * D;
  if (p0 == 0) {
#pragma unroll
    for (int i = 0; i < D; ++i) S[i] = 0.f;
  } else {
#pragma unroll
    for (int i = 0; i < D; ++i) S[i] = st[(size_t)i * D + j];
  }
  const float wn = norm_w[j];
  const float Ah = A[h], dtb = dt_bias[h];
  for (int t = 0; t < n; ++t) {
    const int row = r0 + t;
    const float* xr = qkv + (size_t)row * C;
    const float q = xr[kh * D + j];
    const float k = xr[nk * D + kh * D + j];
    const float v = xr[2 * nk * D + h * D + j];
    const float2 nn = block_sum2_128(q * q, k * k, red);
    qs[j] = q * rsqrtf(nn.x + 1e-6f) * scale;
    ks[j] = k * rsqrtf(nn.y + 1e-6f);
    const float bl = gba.get(row, h), al = gba.get(row, nv + h) + dtb;
    const float beta = 1.f / (1.f + __expf(-bl));
    const float sp = al > 20.f ? al : log1pf(__expf(al));
    const float eg = __expf(Ah * sp);
    __syncthreads();
    float kv = 0.f;
#pragma unroll
    for (int i = 0; i < D; ++i) {
      S[i] *= eg;
      kv += S[i] * ks[i];
    }
    const float dlt = (v - kv) * beta;
    float o = 0.f;
#pragma unroll
    for (int i = 0; i < D; ++i) {
      S[i] += ks[i] * dlt;
      o += S[i] * qs[i];
    }
    const float2 on = block_sum2_128(o * o, 0.f, red);
    const float z = gz.get(row, h * D + j);
    out[(size_t)row * nv * D + h * D + j] =
        __float2half_rn(o * rsqrtf(on.x / D + eps) * wn * silu(z));
  }
#pragma unroll
  for (int i = 0; i < D; ++i) st[(size_t)i * D + j] = S[i];
}

}  // namespace swarm

using namespace swarm;

int launch_ssm_conv_silu(const GemmOut& g, const float* w, int C, int K, float* state,
                         const void* seqs, int S, float* out, cudaStream_t s) {
  if (S <= 0) return 0;
  if (K != 4) return -1;
  dim3 grid((C + 127) / 128, S);
  ssm_conv_silu_kernel<4><<<grid, 128, 0, s>>>(g, w, C, state, (const int4*)seqs, out);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -2;
}

int launch_delta_rule(const float* qkv, int C, int nk, int nv, int D, const GemmOut& gba,
                      const float* dt_bias, const float* A, const GemmOut& gz,
                      const float* norm_w, float eps, float* state, const void* seqs, int S,
                      __half* out, cudaStream_t s) {
  if (S <= 0) return 0;
  if (D != 128 || nv % nk) return -1;
  dim3 grid(S, nv);
  delta_rule_kernel<128><<<grid, 128, 0, s>>>(qkv, C, nk, nv, gba, dt_bias, A, gz, norm_w, eps,
                                              state, (const int4*)seqs, out);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -2;
}
