// Tree ranking for speculative decoding: per row of logits [rows, V], the
// log-sum-exp and the top-k tokens with their log-probabilities -- what the
// drafter needs to grow a tree level (k <= 16).
//
// Two stages so that a handful of rows over a 128k-200k vocabulary still fills
// the GPU:
//   tree_rank_partial  grid (row, slice): each thread keeps a sorted top-K of
//                      its elements in registers plus an online (max, sum-exp);
//                      the CTA merges them (K rounds of a block argmax) and
//                      writes the slice's top-K and (max, sum-exp)
//   tree_rank_merge    one CTA per row: top-k over the slices' candidates and
//                      the combined log-sum-exp -> ids, logit - LSE
// Ties go to the lower token id.
//
// Reference: kernels/tree_rank.cu:230 (tree_rank_partials), :287
// (tree_rank_merge), :426/:486 (top-k partials / merge).
#include "kernels.h"
#include "common.cuh"

namespace swarm {

constexpr int kRankThreads = 256;

SW_DEVICE bool rank_better(float a, int ia, float b, int ib) {
  return a > b || (a == b && ia < ib);
}

// Block-wide best (value, id) among one candidate per thread.
SW_DEVICE void rank_block_best(float v, int id, float* sv, int* si, float& bv, int& bi) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, id, o);
    if (rank_better(ov, oi, v, id)) { v = ov; id = oi; }
  }
  if (lane == 0) { sv[wid] = v; si[wid] = id; }
  __syncthreads();
  if (wid == 0) {
    float x = lane < kRankThreads / 32 ? sv[lane] : -INFINITY;
    int xi = lane < kRankThreads / 32 ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, x, o);
      const int oi = __shfl_xor_sync(0xffffffffu, xi, o);
      if (rank_better(ov, oi, x, xi)) { x = ov; xi = oi; }
    }
    if (lane == 0) { sv[0] = x; si[0] = xi; }
  }
  __syncthreads();
  bv = sv[0];
  bi = si[0];
  __syncthreads();
}

template <int K>
__global__ void __launch_bounds__(kRankThreads) tree_rank_partial_kernel(
    const float* __restrict__ logits, int V, int stride, int slice, int k,
    float* __restrict__ cand_v, int* __restrict__ cand_i, float2* __restrict__ ms) {
  __shared__ float sv[32];
  __shared__ int si[32];
  const int row = blockIdx.x, sl = blockIdx.y, S = gridDim.y;
  const float* r = logits + (size_t)row * stride;
  const int lo = sl * slice, hi = min(V, lo + slice);
  float tv[K];
  int ti[K];
#pragma unroll
  for (int j = 0; j < K; ++j) { tv[j] = -INFINITY; ti[j] = 0x7fffffff; }
  float m = -INFINITY, s = 0.f;
  // four independent loads per step; the running (max, sum-exp) is rescaled
  // once per step instead of once per element
  for (int i0 = lo + threadIdx.x; i0 < hi; i0 += 4 * kRankThreads) {
    float x[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = i0 + u * kRankThreads;
      x[u] = i < hi ? r[i] : -INFINITY;
    }
    const float m4 = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
    if (m4 > m) { s *= __expf(m - m4); m = m4; }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = i0 + u * kRankThreads;
      if (i >= hi) continue;
      if (m > -INFINITY) s += __expf(x[u] - m);
      if (rank_better(x[u], i, tv[K - 1], ti[K - 1])) {  // insert, keep descending order
        float cv = x[u];
        int ci = i;
#pragma unroll
        for (int j = 0; j < K; ++j) {
          if (rank_better(cv, ci, tv[j], ti[j])) {
            const float t1 = tv[j];
            const int t2 = ti[j];
            tv[j] = cv; ti[j] = ci;
            cv = t1; ci = t2;
          }
        }
      }
    }
  }
  // ---- slice (max, sum-exp)
  float gm = m;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, o));
  {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    if (lane == 0) sv[wid] = gm;
    __syncthreads();
    float bm = -INFINITY;
    for (int w = 0; w < kRankThreads / 32; ++w) bm = fmaxf(bm, sv[w]);
    __syncthreads();
    float part = (m == -INFINITY) ? 0.f : s * __expf(m - bm);
    part = warp_sum(part);
    if (lane == 0) sv[wid] = part;
    __syncthreads();
    if (threadIdx.x == 0) {
      float tot = 0.f;
      for (int w = 0; w < kRankThreads / 32; ++w) tot += sv[w];
      ms[(size_t)row * S + sl] = make_float2(bm, tot);
    }
    __syncthreads();
  }
  // ---- slice top-k: k rounds of the block best among each thread's head
  int h = 0;
  for (int j = 0; j < k; ++j) {
    float cv = -INFINITY;
    int ci = 0x7fffffff;
#pragma unroll
    for (int q = 0; q < K; ++q)
      if (q == h) { cv = tv[q]; ci = ti[q]; }
    float bv;
    int bi;
    rank_block_best(cv, ci, sv, si, bv, bi);
    if (ci == bi && bi != 0x7fffffff) ++h;
    if (threadIdx.x == 0) {
      cand_v[((size_t)row * S + sl) * k + j] = bv;
      cand_i[((size_t)row * S + sl) * k + j] = bi;
    }
  }
}

__global__ void __launch_bounds__(kRankThreads) tree_rank_merge_kernel(
    const float* __restrict__ cand_v, const int* __restrict__ cand_i,
    const float2* __restrict__ ms, int S, int k, int32_t* __restrict__ ids,
    float* __restrict__ logp) {
  __shared__ float sv[32];
  __shared__ int si[32];
  __shared__ float lse_s;
  const int row = blockIdx.x;
  const int n = S * k;
  if (threadIdx.x == 0) {
    float M = -INFINITY;
    for (int j = 0; j < S; ++j) M = fmaxf(M, ms[(size_t)row * S + j].x);
    float tot = 0.f;
    for (int j = 0; j < S; ++j) {
      const float2 p = ms[(size_t)row * S + j];
      if (p.x != -INFINITY) tot += p.y * __expf(p.x - M);
    }
    lse_s = M + logf(tot);
  }
  __syncthreads();
  const float lse = lse_s;
  // each thread owns candidates c = tid, tid + 256, ... (n <= 1024 -> at most 4)
  constexpr int kPer = 4;
  float v[kPer];
  int ix[kPer];
#pragma unroll
  for (int q = 0; q < kPer; ++q) {
    const int c = threadIdx.x + q * kRankThreads;
    v[q] = c < n ? cand_v[(size_t)row * n + c] : -INFINITY;
    ix[q] = c < n ? cand_i[(size_t)row * n + c] : 0x7fffffff;
  }
  for (int j = 0; j < k; ++j) {
    float cv = -INFINITY;
    int ci = 0x7fffffff, cq = -1;
#pragma unroll
    for (int q = 0; q < kPer; ++q)
      if (rank_better(v[q], ix[q], cv, ci)) { cv = v[q]; ci = ix[q]; cq = q; }
    float bv;
    int bi;
    rank_block_best(cv, ci, sv, si, bv, bi);
    if (cq >= 0 && ci == bi) {
#pragma unroll
      for (int q = 0; q < kPer; ++q)
        if (q == cq) { v[q] = -INFINITY; ix[q] = 0x7fffffff; }
    }
    if (threadIdx.x == 0) {
      ids[(size_t)row * k + j] = bi;
      logp[(size_t)row * k + j] = bv - lse;
    }
  }
}

}  // namespace swarm

using namespace swarm;

int tree_rank_slices(int rows, int V) {
  // about eight 256-thread CTAs per SM (148 SMs), slices of at least 2048 logits
  int S = rows >= 1184 ? 1 : (1184 + rows - 1) / rows;
  S = S > 64 ? 64 : S;
  const int per = (V + S - 1) / S;
  if (per < 2048) S = (V + 2047) / 2048 > 0 ? (V + 2047) / 2048 : 1;
  return S > 64 ? 64 : S;
}

int launch_tree_rank(const float* logits, int rows, int V, int stride, int k, float* cand_v,
                     int* cand_i, float* ms, int S, int32_t* ids, float* logp, cudaStream_t s) {
  if (rows <= 0) return 0;
  if (k < 1 || k > 16 || S < 1 || S * k > 1024) return -1;
  const int slice = (V + S - 1) / S;
  dim3 grid(rows, S);
  if (k <= 4)
    tree_rank_partial_kernel<4><<<grid, kRankThreads, 0, s>>>(logits, V, stride, slice, k, cand_v,
                                                             cand_i, (float2*)ms);
  else if (k <= 8)
    tree_rank_partial_kernel<8><<<grid, kRankThreads, 0, s>>>(logits, V, stride, slice, k, cand_v,
                                                             cand_i, (float2*)ms);
  else
    tree_rank_partial_kernel<16><<<grid, kRankThreads, 0, s>>>(logits, V, stride, slice, k,
                                                              cand_v, cand_i, (float2*)ms);
  tree_rank_merge_kernel<<<rows, kRankThreads, 0, s>>>(cand_v, cand_i, (const float2*)ms, S, k,
                                                       ids, logp);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -2;
}
