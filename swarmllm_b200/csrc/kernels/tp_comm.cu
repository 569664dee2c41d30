// Tensor parallelism: the reduction of a row-parallel GEMM (o_proj, down_proj)
// fused with the residual add, the next RMSNorm and the all-gather of the
// residual stream, over NVLink peer memory.
//
// A layer's row-parallel GEMM on rank r multiplies its K-slice of the weight
// and produces a partial of the full hidden-wide result.  Its epilogue
// (qgemm_tc.cu / qgemv_q4k.cu, owner_tiles > 0) stores each 128-column tile
// of partials only into the receive buffer of the rank that OWNS those hidden
// columns (rank o owns columns [o*H/W, (o+1)*H/W)): a reduce-scatter done by
// the GEMM itself, tile by tile, as the tiles come out of TMEM.  Its last CTA
// raises a "GEMM done" flag in every rank's arena.
//
// tp_reduce_norm_kernel, per token row t, on rank r:
//   1. wait until every rank's GEMM-done flag has reached this call's epoch;
//   2. for the owned columns: sum the W ranks' partials (GemmOut, n_src = W,
//      all local reads), add the bias and the residual, store the new residual
//      into EVERY rank's copy (P2P stores: the all-gather) and publish this
//      slice's sum of squares next to it, then raise the row flag on every rank;
//   3. wait for the row flags of all W ranks (local polls), add the W sums of
//      squares, and normalise the whole row from the local, now complete copy.
// A row is split into C slices handled by C CTAs (C up to 16 for a few rows,
// 1 for prefill chunks), so decode spreads the partial sums over many SMs;
// flags and sums of squares are then per (rank, slice).
// So each row-parallel layer costs one GEMM launch plus one of this kernel,
// and every byte that crosses NVLink is a store: a partial tile once to its
// owner, a residual slice once to each rank.  Nothing is pulled from a peer.
//
// Buffers alternate between consecutive calls (parity k % 2 of the call
// index): partials buffer, residual copy written, sums of squares.  Call k
// reads the residual from buffer (k+1) % 2 and writes buffer k % 2.  A rank
// only reaches call k + 2, which overwrites what peers read in call k, after
// call k + 1 saw every peer's row flags, i.e. after every peer finished call k.
// Flags carry epochs that every rank counts in lockstep (device counters,
// advanced by the last CTA of each launch, so CUDA-graph replays advance them
// too); waits compare with (int)(flag - want) >= 0 and give up after a
// deadline, recording an error in the status word instead of hanging.
//
// Rows are handled by a grid-stride loop in ascending order with at most a
// few CTAs per SM, so every CTA that waits is resident and the same rows are
// in flight on every rank.
//
// Reference behaviour replaced: the reference's TP sums f32 partials per layer
// and phase through a star or ring of network messages (src/inference/
// allreduce.rs:63,413,620) and applies the residual and norm afterwards.
#include "kernels.h"

#include <cooperative_groups.h>

#include "common.cuh"
#include "ep_common.cuh"
#include "gemm_out.cuh"
#include "tc_utils.cuh"

namespace swarm {

struct TpReduceArgs {
  GemmOut g;                    // this rank's receive buffer, n_src = W sources
  const float* bias;            // [H] or null (added once, by the column's owner)
  const float* w;               // RMSNorm weight [H], or null: no normalised output
  __half* out;                  // [T][out_stride] fp16 normalised rows
  int out_stride;
  float eps;
  int H, W, rank, T, t_stride;  // t_stride: rows of the arena's residual / flag arrays
  int C;                        // CTAs per row: each owns 1/C of the rank's columns
  unsigned long long bases[8];  // every rank's arena base (own included)
  long long h_in_off;           // residual rows read (this rank's copy)
  long long h_out_off;          // residual rows written into every rank
  long long ss_off;             // [W*C][t_stride] fp32 slice sums of squares (this parity)
  long long rowflag_off;        // [W*C][t_stride] u32 slice flags
  const uint32_t* gemm_flags;   // this rank's GEMM-done flags of the receive buffer [W]
  int* ctl_gemm;                // [0]: last GEMM-done epoch waited for (this buffer)
  int* ctl_row;                 // [0]: done-CTA counter, [1]: last row epoch
  int* status;
  int code;
  unsigned long long timeout_ns;
};

SW_DEVICE bool wait_ge(const uint32_t* p, uint32_t want, unsigned long long t0,
                       unsigned long long timeout_ns) {
  int n = 0;
  while ((int)(ld_acquire_sys(p) - want) < 0) {
    if ((++n & 63) == 0 && tc::globaltimer() - t0 > timeout_ns) return false;
  }
  return true;
}

SW_DEVICE void record_fail(int* status, int code, int d0, int d1, int d2) {
  if (status && atomicCAS(&status[0], 0, code) == 0) {
    status[1] = blockIdx.x;
    status[2] = d0;
    status[3] = d1;
    status[4] = d2;
  }
}

SW_DEVICE float4 add4(float4 a, float4 b) {
  return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}

// Work unit u = t * C + j: slice j of row t.  Phase 2 (reduce + publish) covers
// the rank's own columns of the slice, phase 3 (normalise) 1/C of the whole row.
__global__ void __launch_bounds__(256) tp_reduce_norm_kernel(const TpReduceArgs a) {
  pdl_trigger();  // dependents (the next GEMM) may launch and prefetch weights
  pdl_wait();     // what earlier kernels wrote is complete and visible
  __shared__ float red[32];
  __shared__ int ok_s;
  const int H = a.H, W = a.W, C = a.C;
  const uint32_t want_g = (uint32_t)a.ctl_gemm[0] + 1;
  const uint32_t e = (uint32_t)a.ctl_row[1] + 1;
  const unsigned long long t0 = tc::globaltimer();
  if (threadIdx.x == 0) ok_s = 1;
  __syncthreads();
  // 1. every rank's partial tiles for our columns have landed
  if (threadIdx.x < W && !wait_ge(a.gemm_flags + threadIdx.x, want_g, t0, a.timeout_ns)) {
    ok_s = 0;
    record_fail(a.status, a.code, threadIdx.x, (int)want_g, -1);
  }
  __syncthreads();
  const bool ok = ok_s != 0;
  const int per = H / (W * C);              // owned columns of one slice
  const unsigned long long own = a.bases[a.rank];
  const int units = a.T * C;
  // 2. owned columns of every slice this CTA handles: reduce, add, publish
  if (ok) {
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      const int t = u / C, j = u - t * C;
      const int c0 = (a.rank * C + j) * per;
      const float* hin = reinterpret_cast<const float*>(own + a.h_in_off) + (size_t)t * H;
      float ss = 0.f;
      for (int i = c0 + 8 * threadIdx.x; i < c0 + per; i += 8 * blockDim.x) {
        float4 lo, hi;
        a.g.get8(t, i, lo, hi);
        lo = add4(lo, *reinterpret_cast<const float4*>(hin + i));
        hi = add4(hi, *reinterpret_cast<const float4*>(hin + i + 4));
        if (a.bias) {
          lo = add4(lo, *reinterpret_cast<const float4*>(a.bias + i));
          hi = add4(hi, *reinterpret_cast<const float4*>(a.bias + i + 4));
        }
        ss += lo.x * lo.x + lo.y * lo.y + lo.z * lo.z + lo.w * lo.w + hi.x * hi.x +
              hi.y * hi.y + hi.z * hi.z + hi.w * hi.w;
        for (int o = 0; o < W; ++o) {
          float* d = reinterpret_cast<float*>(a.bases[o] + a.h_out_off) + (size_t)t * H + i;
          *reinterpret_cast<float4*>(d) = lo;
          *reinterpret_cast<float4*>(d + 4) = hi;
        }
      }
      ss = block_sum(ss, red);
      __threadfence_system();  // this thread's residual stores before the flags below
      __syncthreads();
      if (threadIdx.x < W) {
        const int o = threadIdx.x;
        const size_t slot = (size_t)(a.rank * C + j) * a.t_stride + t;
        reinterpret_cast<float*>(a.bases[o] + a.ss_off)[slot] = ss;
        __threadfence_system();
        st_release_sys(reinterpret_cast<uint32_t*>(a.bases[o] + a.rowflag_off) + slot, e);
      }
    }
  }
  // 3. 1/C of each whole row: wait for every slice of every rank, then normalise
  const int nflags = W * C;
  const int hc = H / C;
  for (int u = blockIdx.x; ok && u < units; u += gridDim.x) {
    const int t = u / C, j = u - t * C;
    for (int f = threadIdx.x; f < nflags; f += blockDim.x) {
      const uint32_t* p = reinterpret_cast<const uint32_t*>(own + a.rowflag_off) +
                          (size_t)f * a.t_stride + t;
      if (!wait_ge(p, e, t0, a.timeout_ns)) {
        ok_s = 0;
        record_fail(a.status, a.code + 1, f, (int)e, t);
      }
    }
    __syncthreads();
    if (!ok_s) break;
    if (a.w == nullptr) continue;
    const float* ssv = reinterpret_cast<const float*>(own + a.ss_off);
    float part = 0.f;
    for (int f = threadIdx.x; f < nflags; f += blockDim.x)
      part += __ldcg(ssv + (size_t)f * a.t_stride + t);
    const float tot = block_sum(part, red);
    const float inv = rsqrtf(tot / (float)H + a.eps);
    const float* h = reinterpret_cast<const float*>(own + a.h_out_off) + (size_t)t * H;
    __half* o = a.out + (size_t)t * a.out_stride;
    for (int i = j * hc + 8 * threadIdx.x; i < (j + 1) * hc; i += 8 * blockDim.x) {
      const float4 v0 = __ldcg(reinterpret_cast<const float4*>(h + i));
      const float4 v1 = __ldcg(reinterpret_cast<const float4*>(h + i + 4));
      const float4 w0 = *reinterpret_cast<const float4*>(a.w + i);
      const float4 w1 = *reinterpret_cast<const float4*>(a.w + i + 4);
      __half2 r[4];
      r[0] = __floats2half2_rn(v0.x * inv * w0.x, v0.y * inv * w0.y);
      r[1] = __floats2half2_rn(v0.z * inv * w0.z, v0.w * inv * w0.w);
      r[2] = __floats2half2_rn(v1.x * inv * w1.x, v1.y * inv * w1.y);
      r[3] = __floats2half2_rn(v1.z * inv * w1.z, v1.w * inv * w1.w);
      *reinterpret_cast<uint4*>(o + i) = *reinterpret_cast<const uint4*>(r);
    }
  }
  // the last CTA advances the epochs (every CTA has read them by then)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int prev = atomicAdd(&a.ctl_row[0], 1);
    if (prev == (int)gridDim.x - 1) {
      a.ctl_row[0] = 0;
      a.ctl_row[1] = (int)e;
      a.ctl_gemm[0] = (int)want_g;
    }
  }
}

// One-hop variant for few rows (decode): the row-parallel GEMM stored its
// partial tiles into EVERY rank's receive buffer, so each rank sums all W
// partials of every column itself -- the same additions in the same order on
// every rank, so the replicated residual stays bitwise identical -- and the
// only cross-GPU dependency is the GEMM-done flags.  One row per cluster of
// kTpCluster CTAs (distributed shared memory sums the squares), as the
// single-GPU residual + RMSNorm epilogue.
constexpr int kTpCluster = 8;
namespace cg = cooperative_groups;

struct TpLocalArgs {
  GemmOut g;                 // n_src = W sources in this rank's receive buffer
  float* residual;           // [T][H], updated in place
  const float* bias;
  const float* w;            // RMSNorm weight, or null: residual update only
  __half* out;
  int out_stride;
  float eps;
  int W;
  const uint32_t* gemm_flags;
  int* ctl_gemm;             // [0]: last GEMM-done epoch waited for
  int* ctl_done;             // [0]: done-CTA counter
  int* status;
  int code;
  unsigned long long timeout_ns;
};

__global__ void __launch_bounds__(256) tp_local_norm_kernel(const TpLocalArgs a) {
  pdl_trigger();
  pdl_wait();
  cg::cluster_group cluster = cg::this_cluster();
  __shared__ float part;
  __shared__ float red[32];
  __shared__ int ok_s;
  extern __shared__ float slice[];
  const uint32_t want = (uint32_t)a.ctl_gemm[0] + 1;
  const unsigned long long t0 = tc::globaltimer();
  if (threadIdx.x == 0) ok_s = 1;
  __syncthreads();
  if (threadIdx.x < a.W && !wait_ge(a.gemm_flags + threadIdx.x, want, t0, a.timeout_ns)) {
    ok_s = 0;
    record_fail(a.status, a.code, threadIdx.x, (int)want, -2);
  }
  __syncthreads();
  const bool ok = ok_s != 0;
  const int cr = (int)cluster.block_rank(), cn = (int)cluster.num_blocks();
  const int t = blockIdx.x / cn;
  const int dim = a.g.rows;
  const int per = (dim + cn - 1) / cn;
  const int lo = cr * per, hi = min(dim, lo + per);
  float* rr = a.residual + (size_t)t * dim;
  float ss = 0.f;
  if (ok) {
    for (int i = lo + 8 * threadIdx.x; i < hi; i += 8 * blockDim.x) {
      float4 v0, v1;
      a.g.get8(t, i, v0, v1);
      v0 = add4(v0, *reinterpret_cast<const float4*>(rr + i));
      v1 = add4(v1, *reinterpret_cast<const float4*>(rr + i + 4));
      if (a.bias) {
        v0 = add4(v0, *reinterpret_cast<const float4*>(a.bias + i));
        v1 = add4(v1, *reinterpret_cast<const float4*>(a.bias + i + 4));
      }
      *reinterpret_cast<float4*>(rr + i) = v0;
      *reinterpret_cast<float4*>(rr + i + 4) = v1;
      *reinterpret_cast<float4*>(slice + (i - lo)) = v0;
      *reinterpret_cast<float4*>(slice + (i - lo) + 4) = v1;
      ss += v0.x * v0.x + v0.y * v0.y + v0.z * v0.z + v0.w * v0.w + v1.x * v1.x + v1.y * v1.y +
            v1.z * v1.z + v1.w * v1.w;
    }
  }
  ss = block_sum(ss, red);
  if (threadIdx.x == 0) part = ss;
  cluster.sync();
  float tot = 0.f;
  for (int r = 0; r < cn; ++r) tot += *cluster.map_shared_rank(&part, r);
  cluster.sync();  // peers finished reading `part` before any CTA exits
  if (ok && a.out != nullptr && a.w != nullptr) {
    const float inv = rsqrtf(tot / dim + a.eps);
    __half* o = a.out + (size_t)t * a.out_stride;
    for (int i = lo + 8 * threadIdx.x; i < hi; i += 8 * blockDim.x) {
      const float4 v0 = *reinterpret_cast<const float4*>(slice + (i - lo));
      const float4 v1 = *reinterpret_cast<const float4*>(slice + (i - lo) + 4);
      const float4 w0 = *reinterpret_cast<const float4*>(a.w + i);
      const float4 w1 = *reinterpret_cast<const float4*>(a.w + i + 4);
      __half2 r[4];
      r[0] = __floats2half2_rn(v0.x * inv * w0.x, v0.y * inv * w0.y);
      r[1] = __floats2half2_rn(v0.z * inv * w0.z, v0.w * inv * w0.w);
      r[2] = __floats2half2_rn(v1.x * inv * w1.x, v1.y * inv * w1.y);
      r[3] = __floats2half2_rn(v1.z * inv * w1.z, v1.w * inv * w1.w);
      *reinterpret_cast<uint4*>(o + i) = *reinterpret_cast<const uint4*>(r);
    }
  }
  // the last CTA advances the wait epoch (every CTA has read it by then)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int prev = atomicAdd(&a.ctl_done[0], 1);
    if (prev == (int)gridDim.x - 1) {
      a.ctl_done[0] = 0;
      a.ctl_gemm[0] = (int)want;
    }
  }
}

}  // namespace swarm

using namespace swarm;

int launch_tp_local_norm(const GemmOut& g, float* residual, const float* bias, const float* w,
                         __half* out, int out_stride, float eps, int W, const void* gemm_flags,
                         int* ctl_gemm, int* ctl_done, int* status, int code,
                         long long timeout_ns, cudaStream_t s) {
  if (g.T <= 0) return 0;
  const int dim = g.rows;
  if (W < 1 || W > 8 || g.n_src != W || dim % (8 * kTpCluster) != 0) return -1;
  if (out && ((out_stride % 8) != 0 || (reinterpret_cast<uintptr_t>(out) & 15) != 0)) return -3;
  TpLocalArgs a{};
  a.g = g;
  a.residual = residual;
  a.bias = bias;
  a.w = w;
  a.out = out;
  a.out_stride = out_stride ? out_stride : dim;
  a.eps = eps;
  a.W = W;
  a.gemm_flags = static_cast<const uint32_t*>(gemm_flags);
  a.ctl_gemm = ctl_gemm;
  a.ctl_done = ctl_done;
  a.status = status;
  a.code = code;
  a.timeout_ns = timeout_ns > 0 ? (unsigned long long)timeout_ns : tc::kWaitTimeoutNs;
  const int per = dim / kTpCluster;
  if ((size_t)per * sizeof(float) > 48 * 1024 &&
      cudaFuncSetAttribute(tp_local_norm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)(per * sizeof(float))) != cudaSuccess)
    return -4;
  if (launch_pdl_cluster(tp_local_norm_kernel, dim3(g.T * kTpCluster), dim3(256),
                         (size_t)per * sizeof(float), s, kTpCluster, a) != cudaSuccess)
    return -4;
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}

int tp_reduce_slices(int T, int H, int W, int num_sms) {
  // CTAs per row: fill about two CTAs per SM, each slice a whole number of
  // 8-column groups of the rank's columns
  int c = 1;
  while (c < 16 && T * (2 * c) <= 2 * num_sms && (H / W) % (8 * 2 * c) == 0) c *= 2;
  return c;
}

int launch_tp_reduce_norm(const GemmOut& g, const float* bias, const float* w, __half* out,
                          int out_stride, float eps, int H, int W, int rank, int T, int t_stride,
                          const unsigned long long* bases, long long h_in_off, long long h_out_off,
                          long long ss_off, long long rowflag_off, const void* gemm_flags,
                          int* ctl_gemm, int* ctl_row, int* status, int code, int num_sms,
                          long long timeout_ns, cudaStream_t s) {
  if (T <= 0) return 0;
  if (W < 1 || W > 8 || rank < 0 || rank >= W || T > t_stride) return -1;
  if (H % (8 * W) != 0 || g.n_src != W || g.rows != H) return -2;
  const int C = tp_reduce_slices(T, H, W, num_sms);
  if (w && (!out || (out_stride % 8) != 0 || (reinterpret_cast<uintptr_t>(out) & 15) != 0))
    return -3;
  TpReduceArgs a{};
  a.g = g;
  a.bias = bias;
  a.w = w;
  a.out = out;
  a.out_stride = out_stride;
  a.eps = eps;
  a.H = H;
  a.W = W;
  a.rank = rank;
  a.T = T;
  a.t_stride = t_stride;
  a.C = C;
  for (int i = 0; i < W; ++i) a.bases[i] = bases[i];
  a.h_in_off = h_in_off;
  a.h_out_off = h_out_off;
  a.ss_off = ss_off;
  a.rowflag_off = rowflag_off;
  a.gemm_flags = static_cast<const uint32_t*>(gemm_flags);
  a.ctl_gemm = ctl_gemm;
  a.ctl_row = ctl_row;
  a.status = status;
  a.code = code;
  a.timeout_ns = timeout_ns > 0 ? (unsigned long long)timeout_ns : tc::kWaitTimeoutNs;
  // at most 2 CTAs per SM: every CTA resident, rows in ascending order on every rank
  const int units = T * C;
  const int grid = units < 2 * num_sms ? units : 2 * num_sms;
  launch_pdl(tp_reduce_norm_kernel, dim3(grid), dim3(256), 0, s, a);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}
