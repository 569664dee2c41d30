// Gated DeltaNet (linear attention of the Qwen3-Next-style hybrid) on sm_100a.
//
//   ssm_conv_silu   causal depthwise conv1d (kernel 4) over the q|k|v channels
//                   of the in-projection, then SiLU: one thread per (row,
//                   channel), the inputs before the step come from the
//                   per-sequence carried window, which a second kernel then
//                   advances.  Rows of one sequence are consecutive in the batch.
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

// Sequence of batch row r (seqs sorted by row0); -1 if r belongs to none.
SW_DEVICE int seq_of_row(const int4* seqs, int S, int r) {
  int lo = 0, hi = S - 1, f = -1;
  while (lo <= hi) {
    const int m = (lo + hi) >> 1;
    if (seqs[m].x <= r) { f = m; lo = m + 1; } else { hi = m - 1; }
  }
  if (f < 0 || r >= seqs[f].x + seqs[f].y) return -1;
  return f;
}

// One thread per (row, channel); inputs before the sequence's first row of
// this step come from the carried window (zeros at position 0).
template <int K>
__global__ void ssm_conv_silu_kernel(GemmOut g, const float* __restrict__ w, int C,
                                     const float* __restrict__ state,
                                     const int4* __restrict__ seqs, int S,
                                     float* __restrict__ out) {
  pdl_trigger();  // dependents (the next GEMM) may launch and prefetch weights
  pdl_wait();     // what earlier kernels wrote is complete and visible
  const int r = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const int si = seq_of_row(seqs, S, r);
  if (si < 0) return;
  const int4 sq = seqs[si];
  const int l = r - sq.x;
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < K; ++i) {
    const int j = l - (K - 1) + i;  // local index of the input
    float x;
    if (j >= 0) x = g.get(sq.x + j, c);
    else x = sq.w == 0 ? 0.f : state[((size_t)sq.z * (K - 1) + (K - 1) + j) * C + c];
    acc += w[(size_t)c * K + i] * x;
  }
  out[(size_t)r * C + c] = silu(acc);
}

// After the conv: each sequence's window <- its last K-1 inputs.
template <int K>
__global__ void ssm_conv_state_kernel(GemmOut g, int C, float* __restrict__ state,
                                      const int4* __restrict__ seqs) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int4 sq = seqs[blockIdx.y];
  if (c >= C || sq.y <= 0) return;
  float* st = state + (size_t)sq.z * (K - 1) * C;
  float nw[K - 1];
#pragma unroll
  for (int i = 0; i < K - 1; ++i) {
    const int j = sq.y - (K - 1) + i;
    nw[i] = j >= 0 ? g.get(sq.x + j, c) : (sq.w == 0 ? 0.f : st[(size_t)((K - 1) + j) * C + c]);
  }
#pragma unroll
  for (int i = 0; i < K - 1; ++i) st[(size_t)i * C + c] = nw[i];
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
  pdl_trigger();  // dependents (the next GEMM) may launch and prefetch weights
  pdl_wait();     // what earlier kernels wrote is complete and visible
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
  if (S <= 0 || g.T <= 0) return 0;
  if (K != 4) return -1;
  ssm_conv_silu_kernel<4><<<dim3((C + 127) / 128, g.T), 128, 0, s>>>(g, w, C, state,
                                                                      (const int4*)seqs, S, out);
  ssm_conv_state_kernel<4><<<dim3((C + 127) / 128, S), 128, 0, s>>>(g, C, state,
                                                                   (const int4*)seqs);
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
