// Paged decode attention on CUDA cores (split-KV, GQA-grouped), plus the
// log-sum-exp combine that also folds in learned attention sinks.
//
// One CTA = one query row x one KV head (all n_rep query heads of the group)
// x one split (a contiguous run of keys).  Supports: GQA, sliding window,
// learned sinks (gpt-oss), Gemma-style logit softcap, and draft-tree rows
// (keys at or after `tree_start` are visible only if their bit is set in the
// row's 64-bit ancestor mask).
//
// Replaces the reference's decode_attn_f16kv + decode_attn_combine_f32
// (kernels/decode_attn.cu:109,612), which read a contiguous per-request cache;
// this one reads 16-token fp16 pages through a block table.
//
// Cache layout: [pages][n_kv][page_size][head_dim] fp16.
#include "kernels.h"
#include "common.cuh"

namespace swarm {

struct DecodeAttnArgs {
  const __half* q;      // [T, n_q, d]
  const __half* k_cache;
  const __half* v_cache;
  const int32_t* block_table;  // [T, bt_stride]
  int bt_stride;
  const int32_t* seq_lens;     // [T] visible keys (tree rows: prefix + tree nodes)
  const uint64_t* tree_mask;   // [T] or null
  const int32_t* tree_start;   // [T] or null (first tree key position)
  const float* sinks;          // [n_q] or null
  int n_q, n_kv, head_dim, page_size;
  int window;                  // 0 = full
  float scale, softcap;
  int keys_per_split;
  int n_splits;
  float* part_o;               // [T, n_q, n_splits, d]
  float* part_ml;              // [T, n_q, n_splits, 2]
  __half* out;          // [T, n_q, d]
};

template <int D, int NREP>
__global__ void __launch_bounds__(128) decode_attn_split_kernel(DecodeAttnArgs a) {
  pdl_trigger();  // dependents (the next GEMM) may launch and prefetch weights
  pdl_wait();     // what earlier kernels wrote is complete and visible
  const int t = blockIdx.x, hk = blockIdx.y, sp = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int L = a.seq_lens[t];
  int k_begin = sp * a.keys_per_split;
  int k_end = min(L, k_begin + a.keys_per_split);
  const int lo = (a.window > 0) ? max(0, L - a.window) : 0;
  k_begin = max(k_begin, lo);
  extern __shared__ float smem[];
  float* qs = smem;                       // [NREP][D]
  float* sc = qs + NREP * D;              // [NREP][keys_per_split]
  __shared__ float red[32];
  const size_t ml_base = ((size_t)t * a.n_q + hk * NREP) * a.n_splits + sp;
  if (k_begin >= k_end) {
    // Empty split: mark it so the combine skips it.
    if (tid < NREP) {
      a.part_ml[(ml_base + (size_t)tid * a.n_splits) * 2 + 0] = -INFINITY;
      a.part_ml[(ml_base + (size_t)tid * a.n_splits) * 2 + 1] = 0.f;
    }
    return;
  }
  for (int i = tid; i < NREP * D; i += 128)
    qs[i] = __half2float(a.q[((size_t)t * a.n_q + hk * NREP) * D + i]) * a.scale;
  __syncthreads();
  const int32_t* bt = a.block_table + (size_t)t * a.bt_stride;
  const uint64_t tmask = a.tree_mask ? a.tree_mask[t] : ~0ull;
  const int tstart = a.tree_start ? a.tree_start[t] : 0x7fffffff;
  const int nk = k_end - k_begin;
  // dims per lane: D / 32 for D = 64, 128, 256; 4 for D = 96 (lanes 24..31 idle)
  constexpr int PER_LANE = (D % 64 == 0) ? D / 32 : 4;
  const bool lane_on = lane * PER_LANE < D;
  // Phase 1: scores.  A warp takes one key at a time: coalesced 2*D-byte row.
  for (int j = warp; j < nk; j += 4) {
    const int key = k_begin + j;
    const int page = bt[key / a.page_size], off = key % a.page_size;
    const __half* kr = a.k_cache + (((size_t)page * a.n_kv + hk) * a.page_size + off) * D;
    float kf[PER_LANE];
#pragma unroll
    for (int e = 0; e < PER_LANE; e += 2) {
      float2 f = make_float2(0.f, 0.f);
      if (lane_on) f = __half22float2(*reinterpret_cast<const __half2*>(kr + lane * PER_LANE + e));
      kf[e] = f.x;
      kf[e + 1] = f.y;
    }
    bool vis = true;
    if (key >= tstart) vis = (key - tstart) < 64 && ((tmask >> (key - tstart)) & 1ull);
#pragma unroll
    for (int h = 0; h < NREP; ++h) {
      float p = 0.f;
      if (lane_on) {
#pragma unroll
        for (int e = 0; e < PER_LANE; ++e) p = fmaf(qs[h * D + lane * PER_LANE + e], kf[e], p);
      }
      p = warp_sum(p);
      if (a.softcap > 0.f) p = a.softcap * tanhf(p / a.softcap);
      if (lane == 0) sc[h * a.keys_per_split + j] = vis ? p : -INFINITY;
    }
  }
  __syncthreads();
  // Phase 2: softmax statistics per head (one warp per head, round robin).
  __shared__ float mh[NREP], lh[NREP];
  for (int h = warp; h < NREP; h += 4) {
    float m = -INFINITY;
    for (int j = lane; j < nk; j += 32) m = fmaxf(m, sc[h * a.keys_per_split + j]);
    m = warp_max(m);
    float l = 0.f;
    for (int j = lane; j < nk; j += 32) {
      float s = sc[h * a.keys_per_split + j];
      float p = (s == -INFINITY) ? 0.f : __expf(s - m);
      sc[h * a.keys_per_split + j] = p;
      l += p;
    }
    l = warp_sum(l);
    if (lane == 0) { mh[h] = m; lh[h] = l; }
  }
  __syncthreads();
  // Phase 3: P.V; each thread owns D/128*2 ... one dim pair per thread for D<=256.
  for (int dp = tid; dp < D / 2; dp += 128) {
    float acc0[NREP], acc1[NREP];
#pragma unroll
    for (int h = 0; h < NREP; ++h) { acc0[h] = 0.f; acc1[h] = 0.f; }
    for (int j = 0; j < nk; ++j) {
      const int key = k_begin + j;
      const int page = bt[key / a.page_size], off = key % a.page_size;
      const __half* vr = a.v_cache + (((size_t)page * a.n_kv + hk) * a.page_size + off) * D;
      float2 v = __half22float2(*reinterpret_cast<const __half2*>(vr + 2 * dp));
#pragma unroll
      for (int h = 0; h < NREP; ++h) {
        const float p = sc[h * a.keys_per_split + j];
        acc0[h] = fmaf(p, v.x, acc0[h]);
        acc1[h] = fmaf(p, v.y, acc1[h]);
      }
    }
#pragma unroll
    for (int h = 0; h < NREP; ++h) {
      float* po = a.part_o + ((ml_base + (size_t)h * a.n_splits) * D);
      po[2 * dp] = acc0[h];
      po[2 * dp + 1] = acc1[h];
    }
  }
  if (tid < NREP) {
    a.part_ml[(ml_base + (size_t)tid * a.n_splits) * 2 + 0] = mh[tid];
    a.part_ml[(ml_base + (size_t)tid * a.n_splits) * 2 + 1] = lh[tid];
  }
}

// One CTA per (row, q head).  out = sum_s e^{m_s-M} o_s / (sum_s e^{m_s-M} l_s + e^{sink-M}).
__global__ void decode_attn_combine_kernel(const float* __restrict__ part_o,
                                           const float* __restrict__ part_ml, int n_splits, int D,
                                           const float* __restrict__ sinks, int n_q,
                                           __half* __restrict__ out) {
  pdl_trigger();  // dependents (the next GEMM) may launch and prefetch weights
  pdl_wait();     // what earlier kernels wrote is complete and visible
  const int row = blockIdx.x;  // t * n_q + h
  const int h = row % n_q;
  const float* ml = part_ml + (size_t)row * n_splits * 2;
  float M = -INFINITY;
  for (int s = 0; s < n_splits; ++s) M = fmaxf(M, ml[2 * s]);
  const float sink = sinks ? sinks[h] : -INFINITY;
  M = fmaxf(M, sink);
  float denom = (sink == -INFINITY) ? 0.f : __expf(sink - M);
  for (int s = 0; s < n_splits; ++s)
    if (ml[2 * s] != -INFINITY) denom += __expf(ml[2 * s] - M) * ml[2 * s + 1];
  const float inv = denom > 0.f ? 1.f / denom : 0.f;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < n_splits; ++s)
      if (ml[2 * s] != -INFINITY)
        acc += __expf(ml[2 * s] - M) * part_o[((size_t)row * n_splits + s) * D + d];
    out[(size_t)row * D + d] = __float2half_rn(acc * inv);
  }
}

template <int D>
static int dispatch_nrep(const DecodeAttnArgs& a, int nrep, int T, cudaStream_t s) {
  dim3 grid(T, a.n_kv, a.n_splits);
  const size_t sm = (size_t)nrep * (D + a.keys_per_split) * sizeof(float);
#define SW_CASE(R)                                                                      \
  case R:                                                                               \
    if (sm > 48 * 1024)                                                                 \
      cudaFuncSetAttribute(decode_attn_split_kernel<D, R>,                              \
                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);       \
    launch_pdl(decode_attn_split_kernel<D, R>, grid, dim3(128), sm, s, a);              \
    break;
  switch (nrep) {
    SW_CASE(1) SW_CASE(2) SW_CASE(3) SW_CASE(4) SW_CASE(5) SW_CASE(6) SW_CASE(8)
    SW_CASE(16)
    default: return -1;
  }
#undef SW_CASE
  return 0;
}

}  // namespace swarm

using namespace swarm;

int launch_decode_attn_simt(const __half* q, const __half* k_cache, const __half* v_cache,
                            const int32_t* block_table, int bt_stride, const int32_t* seq_lens,
                            const uint64_t* tree_mask, const int32_t* tree_start,
                            const float* sinks, int T, int n_q, int n_kv, int head_dim,
                            int page_size, int window, float scale, float softcap,
                            int keys_per_split, int n_splits, float* part_o, float* part_ml,
                            __half* out, cudaStream_t s) {
  if (T <= 0) return 0;
  DecodeAttnArgs a{q, k_cache, v_cache, block_table, bt_stride, seq_lens, tree_mask, tree_start,
                   sinks, n_q, n_kv, head_dim, page_size, window, scale, softcap,
                   keys_per_split, n_splits, part_o, part_ml, out};
  const int nrep = n_q / n_kv;
  int rc;
  switch (head_dim) {
    case 64: rc = dispatch_nrep<64>(a, nrep, T, s); break;
    case 96: rc = dispatch_nrep<96>(a, nrep, T, s); break;
    case 128: rc = dispatch_nrep<128>(a, nrep, T, s); break;
    case 256: rc = dispatch_nrep<256>(a, nrep, T, s); break;
    default: return -1;
  }
  if (rc) return rc;
  launch_pdl(decode_attn_combine_kernel, dim3(T * n_q), dim3(128), 0, s, part_o, part_ml,
             n_splits, head_dim, sinks, n_q, out);
  SW_LAUNCH_CHECK();
  return 0;
}

// Merge split-KV partials of any attention kernel (SIMT or tcgen05).
void launch_attn_combine(const float* part_o, const float* part_ml, int rows, int n_splits, int D,
                         const float* sinks, int n_q, __half* out, cudaStream_t s) {
  if (rows <= 0) return;
  launch_pdl(decode_attn_combine_kernel, dim3(rows), dim3(128), 0, s, part_o, part_ml, n_splits,
             D, sinks, n_q, out);
  SW_LAUNCH_CHECK();
}
