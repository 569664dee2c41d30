// Mixture-of-experts FFN on sm_100a: routing, token dispatch, grouped expert
// GEMMs on the 5th-generation tensor cores, and the weighted combine.
//
//   moe_topk     router logits (a tensor-core GEMM result) + bias -> top-k
//                selection, routing weights, per-expert token counts (B8 front)
//   moe_plan     one CTA: per-expert offsets (exclusive scan) and the list of
//                (expert, token-tile) work tiles, all on the device so the
//                whole layer is CUDA-graph capturable
//   moe_scatter  (token, k) pairs -> expert-sorted activation rows, with the
//                destination slot of each row (ret)
//   moe_gemm_tc  grouped GEMM over the tiles: W = one expert's rows (Q4_K
//                dequantized to fp16 or MXFP4 dequantized to bf16 in registers,
//                straight into TMEM), X = the expert's token rows by TMA, fp32
//                accumulators double-buffered in TMEM.  Epilogues:
//                  SWIGLU  gate|up interleaved in groups of 16 rows (a
//                          128-row tile = 64 features) -> act(gate + b, up + b)
//                          -> 16-bit H rows
//                  STORE   (+bias) -> fp32 row to out_ptrs[rank][slot] (the
//                          slot/rank come from ret, so the same epilogue writes
//                          a peer GPU's combine buffer under expert parallelism)
//   moe_combine  y[t] = sum_j w[t,j] * rows[t*k+j] (+ sigmoid-gated shared
//                expert), residual add and the next RMSNorm       (B9 tail)
//
// Reference behaviour: MoeFfn routing / top-k / stacked experts
// (src/inference/layers/moe.rs), expert kernels moe_gemm_gguf_kernel and the
// wmma prefill kernel (vendor/candle/candle-kernels/src/moe/moe_gguf.cu:56,
// moe_wmma_gguf.cu:191), gpt-oss clamped SwiGLU (kernels/fused_decode.cu:68).
#include "kernels.h"
#include "gemm_out.cuh"
#include "qgemm_common.cuh"
#include "quant_blocks.cuh"
#include "tc_utils.cuh"
#include "ep_common.cuh"

#include <type_traits>
#include <cooperative_groups.h>
namespace cg = cooperative_groups;

namespace swarm {
using namespace tc;

constexpr int kMoeFmtQ4K = 0;
constexpr int kMoeFmtMX = 1;
constexpr int kMoeEpiSwiglu = 0;
constexpr int kMoeEpiStore = 1;
constexpr int kMxUnitBytes = 128 * kMxRowBytes;  // 17408

// ============================================================== routing
// Router logits come from a tensor-core GEMM (any GemmOut).  One CTA per
// token: all threads read the (split-K) logits in parallel into shared
// memory, then warp 0 adds nothing more than the selection: top-k (ties ->
// lower expert id), routing weights, per-expert token counts.
// mode 0: softmax over all experts, weights = their probabilities;
// mode 1: top-k on the logits, softmax over the k selected;
// mode 2 (GLM-4.5 / DeepSeek-V3 style): scores sigmoid(logit), top-k on
//   score + sel_b[e] (a selection bias that does not enter the weight),
//   weights = the k scores, divided by their sum when `norm`, times `scale`.
__global__ void __launch_bounds__(256) moe_topk_kernel(GemmOut lg, const float* __restrict__ br,
                                                       int T, int E, int k, int mode,
                                                       const float* __restrict__ sel_b, int norm,
                                                       float scale,
                                                       int32_t* __restrict__ ids,
                                                       float* __restrict__ wts,
                                                       int* __restrict__ counts) {
  __shared__ float lgs[512];
  const int t = blockIdx.x;
  for (int e = threadIdx.x; e < E; e += blockDim.x) lgs[e] = lg.get(t, e) + (br ? br[e] : 0.f);
  __syncthreads();
  if (threadIdx.x >= 32) return;
  const int lane = threadIdx.x;
  constexpr int kMaxPer = 16;  // E <= 512
  const bool sig = mode == 2;
  const int softmax_after_topk = mode == 1;
  float v[kMaxPer];
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < E ? (sig ? 1.f / (1.f + __expf(-lgs[e])) + (sel_b ? sel_b[e] : 0.f) : lgs[e])
                 : -INFINITY;
  }
  float sel_v = 0.f, top = 0.f, denom_all = 0.f;
  int sel_e = 0;
  for (int j = 0; j < k; ++j) {
    float bv = -INFINITY;
    int be = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i)
      if (v[i] > bv) { bv = v[i]; be = lane + 32 * i; }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oe = __shfl_xor_sync(0xffffffffu, be, o);
      if (ov > bv || (ov == bv && oe < be)) { bv = ov; be = oe; }
    }
    if (j == 0 && !sig) {
      top = bv;
      if (!softmax_after_topk) {  // softmax over all experts, then pick
        float sum = 0.f;
#pragma unroll
        for (int i = 0; i < kMaxPer; ++i)
          if (lane + 32 * i < E) sum += __expf(v[i] - top);
        denom_all = warp_sum(sum);
      }
    }
    if (be >= E) be = 0;  // only reachable with NaN logits
    if (lane == j) { sel_v = bv; sel_e = be; }
    if ((be & 31) == lane) {
#pragma unroll
      for (int i = 0; i < kMaxPer; ++i)
        if (lane + 32 * i == be) v[i] = -INFINITY;
    }
  }
  float w;
  if (sig) {  // the selected expert's score without the selection bias
    const float sc = lane < k ? 1.f / (1.f + __expf(-lgs[sel_e])) : 0.f;
    const float sum = warp_sum(sc);
    w = (norm && sum > 0.f ? sc / sum : sc) * scale;
  } else {
    const float ex = lane < k ? __expf(sel_v - top) : 0.f;
    const float denom = softmax_after_topk ? warp_sum(ex) : denom_all;
    w = ex / denom;
  }
  if (lane < k) {
    const size_t o = (size_t)t * k + lane;
    ids[o] = sel_e;
    wts[o] = w;
    atomicAdd(&counts[sel_e], 1);
  }
}

// One CTA of 1024 threads (E <= 1024).  counts -> offsets/cursors, tile list,
// and counts reset to zero for the next layer.
__global__ void __launch_bounds__(1024) moe_plan_kernel(int* __restrict__ counts, int E, int N,
                                                        int* __restrict__ offsets,
                                                        int* __restrict__ cursor,
                                                        int4* __restrict__ tiles,
                                                        int* __restrict__ n_tiles, int max_tiles,
                                                        int* __restrict__ status) {
  __shared__ int s_c[32], s_t[32];
  const int e = threadIdx.x, lane = e & 31, warp = e >> 5;
  const int c = e < E ? counts[e] : 0;
  const int nt = (c + N - 1) / N;
  int ic = c, it = nt;  // inclusive warp scans
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int a = __shfl_up_sync(0xffffffffu, ic, o), b = __shfl_up_sync(0xffffffffu, it, o);
    if (lane >= o) { ic += a; it += b; }
  }
  if (lane == 31) { s_c[warp] = ic; s_t[warp] = it; }
  __syncthreads();
  if (warp == 0) {
    int a = s_c[lane], b = s_t[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int x = __shfl_up_sync(0xffffffffu, a, o), y = __shfl_up_sync(0xffffffffu, b, o);
      if (lane >= o) { a += x; b += y; }
    }
    s_c[lane] = a;
    s_t[lane] = b;
  }
  __syncthreads();
  const int base_c = (warp ? s_c[warp - 1] : 0) + ic - c;
  const int base_t = (warp ? s_t[warp - 1] : 0) + it - nt;
  if (e < E) {
    offsets[e] = base_c;
    cursor[e] = base_c;
    for (int j = 0; j < nt; ++j)
      if (base_t + j < max_tiles)
        tiles[base_t + j] = make_int4(e, base_c + j * N, min(N, c - j * N), 0);
    counts[e] = 0;
  }
  if (e == 1023) {
    const int total_t = s_t[31];
    offsets[E] = s_c[31];
    *n_tiles = min(total_t, max_tiles);
    if (total_t > max_tiles && status) status[6] = total_t;  // capacity bug: reported, tiles dropped
  }
}

// One warp per (token, k) pair: reserve the row, copy the activation row (fp16
// -> fp16 or bf16) and record its slot.
template <typename XT>
__global__ void moe_scatter_kernel(const __half* __restrict__ x, int x_stride, int H,
                                   const int32_t* __restrict__ ids, int P, int k,
                                   int* __restrict__ cursor, XT* __restrict__ xs, int xs_stride,
                                   int32_t* __restrict__ ret, int rank_bits) {
  const int p = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (p >= P || ids[p] < 0) return;  // -1: routed to another rank's expert (TP)
  int pos = 0;
  if (lane == 0) {
    pos = atomicAdd(&cursor[ids[p]], 1);
    ret[pos] = rank_bits | p;
  }
  pos = __shfl_sync(0xffffffffu, pos, 0);
  const __half* src = x + (size_t)(p / k) * x_stride;
  XT* dst = xs + (size_t)pos * xs_stride;
  for (int i = lane * 2; i < H; i += 64) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(src + i));
    dst[i] = from_f<XT>(f.x);
    dst[i + 1] = from_f<XT>(f.y);
  }
}

// ============================================================== grouped GEMM
template <int N, int FMT>
struct MCfg {
  static constexpr int DQ = N <= 64 ? 3 : 2;
  static constexpr int U = DQ;
  static constexpr int THREADS = 96 + 128 * DQ;
  static constexpr int FIRST_DQ_WARP = 3;
  static constexpr int A_COL = 512 - 128 * U;  // two accumulator slots below it
  // Each slot rotates its MMAs over NACC sub-accumulators (summed in the
  // drain): at decode sizes consecutive MMAs into one accumulator wait for
  // each other, independent ones overlap.
  static constexpr int NACC = (A_COL / (2 * N)) >= 4 ? 4 : ((A_COL / (2 * N)) >= 2 ? 2 : 1);
  static constexpr int SLOT = NACC * N;          // TMEM columns per slot
  static_assert(A_COL >= 2 * SLOT, "TMEM budget");
  static constexpr int X_UNIT_BYTES = N * 512;
  static constexpr int W_STAGE = FMT == kMoeFmtQ4K ? 128 * kQ4kRowBytes : kMxUnitBytes;
  static constexpr int W_ST = 2 * DQ;
  static constexpr int X_BYTES = U * X_UNIT_BYTES;
  static constexpr int W_BYTES = W_ST * W_STAGE;
  static constexpr int BAR_BYTES = 512;
  static constexpr int SMEM = 1024 + X_BYTES + W_BYTES + BAR_BYTES;
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
};

struct MoeGemmArgs {
  const uint8_t* w;
  long long w_expert_bytes, w_tile_bytes;
  int w_last_bytes;
  int row_tiles;    // 128-row tiles per expert
  int rows_valid;   // STORE: output rows; SWIGLU: F
  int n_units;      // 256-wide K units (last may be partial)
  int last_k;       // K values in the last unit
  const int4* tiles;
  const int* n_tiles;
  const float* bias;
  int bias_stride;
  void* h;
  int h_stride, act_kind;
  float alpha, limit;
  unsigned long long out_ptrs[8];
  int out_stride;
  const int32_t* ret;
  int* status;
  // optional completion signal to the peers (expert parallelism): ctl[0..1]
  // = done counter, epoch; flag word at sig_bases[o] + sig_flag_off + 4 * rank
  int* sig_ctl;
  unsigned long long sig_bases[8];
  long long sig_flag_off;
  int sig_world, sig_rank;
};

SW_DEVICE float moe_act(float g, float u, int kind, float alpha, float limit) {
  if (kind == 0) return silu(g) * u;
  g = fminf(g, limit);
  u = fminf(fmaxf(u, -limit), limit);
  return g / (1.f + __expf(-alpha * g)) * (u + 1.f);
}

template <int N, int FMT, int EPI>
__global__ void __launch_bounds__(MCfg<N, FMT>::THREADS, 1)
    moe_gemm_tc_kernel(const __grid_constant__ CUtensorMap x_map, MoeGemmArgs a) {
  using C = MCfg<N, FMT>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* x_smem = smem;
  uint8_t* w_smem = smem + C::X_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(w_smem + C::W_BYTES);
  uint64_t* w_full = bars;
  uint64_t* w_empty = w_full + C::W_ST;
  uint64_t* ready = w_empty + C::W_ST;
  uint64_t* empty = ready + C::U;
  uint64_t* d_full = empty + C::U;  // [2]
  uint64_t* d_empty = d_full + 2;   // [2]
  uint64_t* done_bar = d_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int RT = a.row_tiles;
  const int n_items = *a.n_tiles * RT;
  const int n_my = n_items > (int)blockIdx.x ? (n_items - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int total = n_my * a.n_units;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::W_ST; ++i) { mbar_init(&w_full[i], 1); mbar_init(&w_empty[i], 4); }
    for (int i = 0; i < C::U; ++i) { mbar_init(&ready[i], 5); mbar_init(&empty[i], 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(&d_full[i], 1); mbar_init(&d_empty[i], 4); }
    mbar_init(done_bar, 1);
    fence_barrier_init();
    prefetch_tensormap(&x_map);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ W producer
    if (lane == 0) {
      int issued = 0;
      bool ok = true;
      for (int i = 0; i < total && ok; ++i) {
        const int li = i / a.n_units, u = i - li * a.n_units;
        const int it = (int)blockIdx.x + li * (int)gridDim.x;
        const int tile = it / RT, rt = it - tile * RT;
        const int e = a.tiles[tile].x;
        const int wsi = i % C::W_ST;
        if (!(ok = mbar_wait(&w_empty[wsi], ((i / C::W_ST) & 1) ^ 1, a.status, 41, i, 0))) break;
        const uint32_t bytes = (u == a.n_units - 1) ? (uint32_t)a.w_last_bytes : (uint32_t)C::W_STAGE;
        mbar_arrive_expect_tx(&w_full[wsi], bytes);
        bulk_load(w_smem + wsi * C::W_STAGE,
                  a.w + (size_t)e * a.w_expert_bytes + (size_t)rt * a.w_tile_bytes +
                      (size_t)u * C::W_STAGE,
                  bytes, &w_full[wsi]);
        ++issued;
      }
      if (!ok)
        for (int i = max(0, issued - C::W_ST); i < issued; ++i)
          mbar_wait(&w_full[i % C::W_ST], (i / C::W_ST) & 1, nullptr, 0);
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------ X producer
    if (lane == 0) {
      int issued = 0;
      bool ok = true;
      for (int i = 0; i < total && ok; ++i) {
        const int li = i / a.n_units, u = i - li * a.n_units;
        const int it = (int)blockIdx.x + li * (int)gridDim.x;
        const int row0 = a.tiles[it / RT].y;
        const int s = i % C::U;
        if (!(ok = mbar_wait(&empty[s], ((i / C::U) & 1) ^ 1, a.status, 42, i, 0))) break;
        const int kvalid = (u == a.n_units - 1) ? a.last_k : 256;
        const int nbox = (kvalid + 63) >> 6;
        mbar_arrive_expect_tx(&ready[s], nbox * N * 128);
        uint8_t* dst = x_smem + s * C::X_UNIT_BYTES;
        for (int c = 0; c < nbox; ++c)
          tma_load_2d(dst + c * (N * 128), &x_map, u * 256 + c * 64, row0, &ready[s]);
        ++issued;
      }
      if (!ok)
        for (int i = max(0, issued - C::U); i < issued; ++i)
          mbar_wait(&ready[i % C::U], (i / C::U) & 1, nullptr, 0);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(128, N, FMT == kMoeFmtMX ? 1 : 0);
      const uint64_t xdesc0 = smem_desc(smem_u32(x_smem), 16, 1024, 2);
      bool ok = true;
      for (int i = 0; i < total && ok; ++i) {
        const int li = i / a.n_units, u = i - li * a.n_units;
        const bool first = u == 0, last = u == a.n_units - 1;
        const int slot = li & 1;
        if (first && li >= 2) {
          if (!(ok = mbar_wait(&d_empty[slot], ((li >> 1) - 1) & 1, a.status, 43, i, li))) break;
        }
        const int s = i % C::U;
        if (!(ok = mbar_wait(&ready[s], (i / C::U) & 1, a.status, 44, i, 0))) break;
        tc_fence_after();
        const uint64_t xd = xdesc0 + (uint64_t)((s * C::X_UNIT_BYTES) >> 4);
        const uint32_t ab = tmem_base + C::A_COL + s * 128;
        const uint32_t dt = tmem_base + slot * C::SLOT;
        const int nk = (last ? a.last_k : 256) >> 4;
        for (int kk = 0; kk < nk; ++kk)
          umma_f16_ts(dt + (uint32_t)((kk % C::NACC) * N), ab + kk * 8,
                      xd + (uint64_t)((((kk >> 2) * (N * 128)) + (kk & 3) * 32) >> 4), idesc,
                      (first && kk < C::NACC) ? 0u : 1u);
        umma_commit(&empty[s]);
        if (last) umma_commit(&d_full[slot]);
      }
      umma_commit(done_bar);
      mbar_wait(done_bar, 0, nullptr, 0);
    }
  } else {
    // ------------------------------------------------------------ dequant + epilogue
    const int g = (warp - C::FIRST_DQ_WARP) >> 2;
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    bool ok = true;
    for (int i = 0; i < total && ok; ++i) {
      const int li = i / a.n_units, u = i - li * a.n_units;
      const bool last = u == a.n_units - 1;
      if ((i % C::DQ) == g) {
        const int wsi = i % C::W_ST;
        const int s = i % C::U;
        if (!(ok = mbar_wait_warp(&w_full[wsi], (i / C::W_ST) & 1, a.status, 45, i, 0))) break;
        const uint32_t taddr = tmem_base + lane_off + C::A_COL + s * 128;
        if constexpr (FMT == kMoeFmtQ4K) {
          const uint4* src = reinterpret_cast<const uint4*>(w_smem + wsi * C::W_STAGE +
                                                             row * kQ4kRowBytes);
          uint4 q[8];
#pragma unroll
          for (int c = 0; c < 8; ++c) q[c] = src[c];
          const uint4 hdr = src[8];
          __syncwarp();
          if (lane == 0) mbar_arrive(&w_empty[wsi]);
          float sc_f[8], mb_f[8];
          q4k_decode_scales(hdr, sc_f, mb_f);
          if (!(ok = mbar_wait_warp(&empty[s], ((i / C::U) & 1) ^ 1, a.status, 46, i, 0))) break;
          tc_fence_after();
          dq_unit(q, sc_f, mb_f, taddr);
        } else {
          const int nb = last ? (a.last_k >> 5) : 8;
          const uint2* src = reinterpret_cast<const uint2*>(w_smem + wsi * C::W_STAGE +
                                                             row * (8 + 16 * nb));
          const uint2 sc = src[0];
          if (!(ok = mbar_wait_warp(&empty[s], ((i / C::U) & 1) ^ 1, a.status, 46, i, 0))) break;
          tc_fence_after();
#pragma unroll 1
          for (int b = 0; b < nb; ++b) {
            const uint2 q0 = src[1 + 2 * b], q1 = src[2 + 2 * b];
            const uint32_t e8 = ((b < 4 ? sc.x : sc.y) >> (8 * (b & 3))) & 0xFFu;
            const uint32_t s2 = mx_scale_bf16x2(e8);
            uint32_t cols[16];
            dq_mx_word(q0.x, s2, cols);
            dq_mx_word(q0.y, s2, cols + 4);
            dq_mx_word(q1.x, s2, cols + 8);
            dq_mx_word(q1.y, s2, cols + 12);
            tmem_st_x16(taddr + b * 16, cols);
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&w_empty[wsi]);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&ready[s]);
      }
      if (last && g == 0) {
        // Warpgroup 0 drains every item, in order (accumulator slot li & 1).
        const int slot = li & 1;
        if (!(ok = mbar_wait_warp(&d_full[slot], (li >> 1) & 1, a.status, 47, i, li))) break;
        tc_fence_after();
        const int it = (int)blockIdx.x + li * (int)gridDim.x;
        const int tile = it / RT, rt = it - tile * RT;
        const int4 tinfo = a.tiles[tile];
        const int e = tinfo.x, row0 = tinfo.y, nrows = tinfo.z;
        const uint32_t dbase = tmem_base + lane_off + slot * C::SLOT;
        if constexpr (EPI == kMoeEpiStore) {
          const int rowg = rt * 128 + row;
          const bool valid = rowg < a.rows_valid;
          const float bias = (a.bias && valid) ? a.bias[(size_t)e * a.bias_stride + rowg] : 0.f;
#pragma unroll 1
          for (int c = 0; c < N / 16; ++c) {
            uint32_t r[16];
            tmem_ld_x16(dbase + c * 16, r);
            tmem_wait_ld();
#pragma unroll
            for (int acc = 1; acc < C::NACC; ++acc) {
              uint32_t r2[16];
              tmem_ld_x16(dbase + acc * N + c * 16, r2);
              tmem_wait_ld();
#pragma unroll
              for (int e = 0; e < 16; ++e)
                r[e] = __float_as_uint(__uint_as_float(r[e]) + __uint_as_float(r2[e]));
            }
#pragma unroll
            for (int q = 0; q < 16; ++q) {
              const int t = c * 16 + q;
              if (t < nrows && valid) {
                const int dst = a.ret[row0 + t];
                float* o = reinterpret_cast<float*>(a.out_ptrs[(dst >> 24) & 7]);
                o[(size_t)(dst & 0xFFFFFF) * a.out_stride + rowg] = __uint_as_float(r[q]) + bias;
              }
            }
          }
        } else {
          // Rows 32q + [0,16) are gate features rt*64 + 16q + [0,16) and rows
          // 32q + [16,32) the matching up features, so lane l and lane l ^ 16
          // of a warp hold the two halves of one feature: one shuffle pairs
          // them, even tokens go to the gate lane and odd ones to the up lane.
          using HT = typename std::conditional<FMT == kMoeFmtMX, __nv_bfloat16, __half>::type;
          HT* hout = reinterpret_cast<HT*>(a.h);
          const float bias = a.bias ? a.bias[(size_t)e * a.bias_stride + rt * 128 + row] : 0.f;
          const int f = rt * 64 + quad * 16 + (lane & 15);
          const bool is_gate = lane < 16;
#pragma unroll 1
          for (int c = 0; c < N / 16; ++c) {
            uint32_t r[16];
            tmem_ld_x16(dbase + c * 16, r);
            tmem_wait_ld();
#pragma unroll
            for (int acc = 1; acc < C::NACC; ++acc) {
              uint32_t r2[16];
              tmem_ld_x16(dbase + acc * N + c * 16, r2);
              tmem_wait_ld();
#pragma unroll
              for (int e = 0; e < 16; ++e)
                r[e] = __float_as_uint(__uint_as_float(r[e]) + __uint_as_float(r2[e]));
            }
#pragma unroll
            for (int q = 0; q < 16; q += 2) {
              const float v0 = __uint_as_float(r[q]) + bias, v1 = __uint_as_float(r[q + 1]) + bias;
              // gate lane keeps token q and sends token q+1; up lane the reverse
              const float send = is_gate ? v1 : v0;
              const float recv = __shfl_xor_sync(0xffffffffu, send, 16);
              const int t = c * 16 + q + (is_gate ? 0 : 1);
              const float g = is_gate ? v0 : recv, u = is_gate ? recv : v1;
              if (t < nrows && f < a.rows_valid)
                hout[(size_t)(row0 + t) * a.h_stride + f] =
                    from_f<HT>(moe_act(g, u, a.act_kind, a.alpha, a.limit));
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&d_empty[slot]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
  if (a.sig_ctl != nullptr)
    ep_grid_done_signal(a.sig_ctl, a.sig_bases, a.sig_flag_off, a.sig_world, a.sig_rank);
}

// ============================================================== combine
// One CTA per token: v = sum_j w[t,j] * rows[t*k+j] + gate * shared; residual
// += v; optional RMSNorm of the new residual into `out`.
__global__ void __launch_bounds__(512) moe_combine_kernel(
    const float* __restrict__ rows, int row_stride, const float* __restrict__ wts, int k,
    GemmOut sh, int has_sh, GemmOut shg, int has_shg, float* __restrict__ residual, int H,
    const float* __restrict__ norm_w, __half* __restrict__ out, int out_stride, float eps) {
  pdl_trigger();  // dependents (the next GEMM) may launch and prefetch weights
  pdl_wait();     // what earlier kernels wrote is complete and visible
  extern __shared__ float crow[];
  __shared__ float red[32];
  const int t = blockIdx.x;
  float gate = 1.f;
  if (has_shg) gate = 1.f / (1.f + __expf(-shg.get(t, 0)));
  float ss = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    float v = 0.f;
    for (int j = 0; j < k; ++j) v += wts[t * k + j] * rows[(size_t)(t * k + j) * row_stride + i];
    if (has_sh) v += gate * sh.get(t, i);
    const float r = residual[(size_t)t * H + i] + v;
    residual[(size_t)t * H + i] = r;
    crow[i] = r;
    ss += r * r;
  }
  if (out == nullptr) return;
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / H + eps);
  for (int i = threadIdx.x; i < H; i += blockDim.x)
    out[(size_t)t * out_stride + i] = __float2half_rn(crow[i] * inv * norm_w[i]);
}

// ============================================================== tensor parallelism
// Under tensor parallelism every rank of the group holds every token and
// experts [e0, e0 + n_loc).  moe_localize keeps this rank's (token, k) pairs:
// their expert ids become local, the others get id -1 and weight 0; the
// per-expert counts move to [0, n_loc) and the rest are cleared (moe_plan
// expects zero counts on entry of the next layer).  One CTA.
__global__ void moe_localize_kernel(int32_t* __restrict__ ids, float* __restrict__ wts,
                                    int* __restrict__ counts, int P, int E, int e0, int n_loc) {
  __shared__ int sc[1024];
  for (int e = threadIdx.x; e < E; e += blockDim.x) sc[e] = counts[e];
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) counts[e] = e < n_loc ? sc[e0 + e] : 0;
  for (int p = threadIdx.x; p < P; p += blockDim.x) {
    const int e = ids[p];
    if (e >= e0 && e < e0 + n_loc) {
      ids[p] = e - e0;
    } else {
      ids[p] = -1;
      wts[p] = 0.f;
    }
  }
}

// This rank's share of the MoE output, v = sum_j w[t,j] * rows[t*k+j] (its own
// experts; w = 0 for the others) + gate * shared (its slice of the shared
// expert's down projection), stored column block by column block into the
// receive slot of the rank that owns those columns (dst[o] + t * H + c, over
// NVLink for the other ranks); the CTA that finishes last raises this rank's
// done flag on every rank.  tp_reduce_norm then sums the W slots, adds the
// residual and normalises (tp_comm.cu).  One CTA per token.
__global__ void __launch_bounds__(256) moe_combine_tp_kernel(
    const float* __restrict__ rows, int row_stride, const float* __restrict__ wts, int k,
    GemmOut sh, int has_sh, GemmOut shg, int has_shg, int H, int W, EpPeers dst, int* ctl,
    EpPeers sig, long long flag_off, int rank, int to_all) {
  const int t = blockIdx.x;
  const int per = H / W;
  float gate = 1.f;
  if (has_shg) gate = 1.f / (1.f + __expf(-shg.get(t, 0)));
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    float v = 0.f;
    for (int j = 0; j < k; ++j) {
      const float w = wts[t * k + j];
      if (w != 0.f) v += w * rows[(size_t)(t * k + j) * row_stride + i];
    }
    if (has_sh) v += gate * sh.get(t, i);
    if (to_all) {   // every rank sums every column itself (one-hop TP reduce)
      for (int o = 0; o < W; ++o) reinterpret_cast<float*>(dst.base[o])[(size_t)t * H + i] = v;
    } else {
      reinterpret_cast<float*>(dst.base[i / per])[(size_t)t * H + i] = v;
    }
  }
  ep_grid_done_signal(ctl, sig.base, flag_off, W, rank);
}

// ============================================================== repack
// GGUF MXFP4 [rows][K/32 blocks of 17 B] (one expert) -> [row_tiles][units]
// [128 rows][8 + 16 nb] with the nibble order of dq_mx_word.  Padding rows
// are zero.
__global__ void mxfp4_repack_kernel(const uint8_t* __restrict__ src, int rows, int rows_pad, int K,
                                    uint8_t* __restrict__ dst) {
  const int nblk = K / 32;
  const int n_units = (K + 255) / 256;
  const int last_nb = nblk - (n_units - 1) * 8;
  const long long tile_bytes = (long long)(n_units - 1) * kMxUnitBytes + 128LL * (8 + 16 * last_nb);
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)rows_pad * n_units) return;
  const int r = (int)(idx / n_units), u = (int)(idx - (long)r * n_units);
  const int nb = (u == n_units - 1) ? last_nb : 8;
  uint8_t* out = dst + (size_t)(r >> 7) * tile_bytes + (size_t)u * kMxUnitBytes +
                 (size_t)(r & 127) * (8 + 16 * nb);
  for (int b = 0; b < 8; ++b) out[b] = 0;
  if (r >= rows) {
    for (int i = 0; i < 16 * nb; ++i) out[8 + i] = 0;
    return;
  }
  for (int b = 0; b < nb; ++b) {
    const uint8_t* blk = src + ((size_t)r * nblk + u * 8 + b) * 17;
    out[b] = blk[0];
    const uint8_t* qs = blk + 1;
    for (int w = 0; w < 4; ++w) {
      uint32_t word = 0;
      for (int i = 0; i < 4; ++i) {
        const int v0 = 8 * w + 2 * i, v1 = v0 + 1;
        const uint32_t n0 = v0 < 16 ? (qs[v0] & 15) : (qs[v0 - 16] >> 4);
        const uint32_t n1 = v1 < 16 ? (qs[v1] & 15) : (qs[v1 - 16] >> 4);
        word |= (n0 << (4 * i)) | (n1 << (16 + 4 * i));
      }
      reinterpret_cast<uint32_t*>(out + 8 + 16 * b)[w] = word;  // 8 + 16b + 4w: 4-aligned
    }
  }
}

}  // namespace swarm

using namespace swarm;

// ---------------------------------------------------------------- host side
int moe_tok_tile(int pairs, int n_experts) {
  const int active = pairs < n_experts ? pairs : n_experts;
  const int avg = active > 0 ? (pairs + active - 1) / active : 1;
  if (avg <= 16) return 16;
  if (avg <= 32) return 32;
  if (avg <= 64) return 64;
  return 128;
}

int moe_max_tiles(int pairs, int n_experts, int tok_tile) {
  return (pairs + tok_tile - 1) / tok_tile + (pairs < n_experts ? pairs : n_experts);
}

long long moe_packed_bytes(int fmt, int rows, int K) {
  const int rows_pad = (rows + 127) / 128 * 128;
  if (fmt == kMoeFmtQ4K) return (long long)rows_pad * (K / 256) * kQ4kRowBytes;
  const int nblk = K / 32, n_units = (K + 255) / 256, last_nb = nblk - (n_units - 1) * 8;
  return (long long)(rows_pad / 128) *
         ((long long)(n_units - 1) * kMxUnitBytes + 128LL * (8 + 16 * last_nb));
}

int launch_mxfp4_repack(const void* src, int rows, int K, void* dst, cudaStream_t s) {
  if (K % 32) return -1;
  const int rows_pad = (rows + 127) / 128 * 128;
  const long n = (long)rows_pad * ((K + 255) / 256);
  mxfp4_repack_kernel<<<(unsigned)((n + 127) / 128), 128, 0, s>>>((const uint8_t*)src, rows,
                                                                   rows_pad, K, (uint8_t*)dst);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -2;
}

int launch_moe_topk(const GemmOut& lg, const float* br, int T, int E, int k, int mode,
                    const float* sel_b, int norm, float scale, int32_t* ids, float* wts,
                    int* counts, cudaStream_t s) {
  if (T <= 0) return 0;
  if (E > 512 || k > 32 || k > E || mode < 0 || mode > 2) return -1;
  moe_topk_kernel<<<T, 256, 0, s>>>(lg, br, T, E, k, mode, sel_b, norm, scale, ids, wts, counts);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}

int launch_moe_plan(int* counts, int E, int tok_tile, int* offsets, int* cursor, void* tiles,
                    int* n_tiles, int max_tiles, int* status, cudaStream_t s) {
  if (E > 1024) return -1;
  moe_plan_kernel<<<1, 1024, 0, s>>>(counts, E, tok_tile, offsets, cursor, (int4*)tiles, n_tiles,
                                     max_tiles, status);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -2;
}

int launch_moe_scatter(const __half* x, int x_stride, int H, const int32_t* ids, int P, int k,
                       int* cursor, void* xs, int xs_stride, int xs_bf16, int32_t* ret,
                       int rank, cudaStream_t s) {
  if (P <= 0) return 0;
  if (H % 2) return -1;
  const int warps = 8;
  const unsigned grid = (unsigned)((P + warps - 1) / warps);
  const int rb = rank << 24;
  if (xs_bf16)
    moe_scatter_kernel<__nv_bfloat16><<<grid, 32 * warps, 0, s>>>(
        x, x_stride, H, ids, P, k, cursor, (__nv_bfloat16*)xs, xs_stride, ret, rb);
  else
    moe_scatter_kernel<__half><<<grid, 32 * warps, 0, s>>>(x, x_stride, H, ids, P, k, cursor,
                                                           (__half*)xs, xs_stride, ret, rb);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -2;
}

template <int N, int FMT, int EPI>
static int moe_launch_n(const CUtensorMap& map, const MoeGemmArgs& a, int ctas, cudaStream_t s) {
  using C = MCfg<N, FMT>;
  static unsigned long long attr_done = 0;
  if (!smem_attr_once(moe_gemm_tc_kernel<N, FMT, EPI>, C::SMEM, &attr_done)) return -3;
  moe_gemm_tc_kernel<N, FMT, EPI><<<ctas, C::THREADS, C::SMEM, s>>>(map, a);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}

template <int FMT, int EPI>
static int moe_launch_fmt(int N, const CUtensorMap& map, const MoeGemmArgs& a, int ctas,
                          cudaStream_t s) {
  switch (N) {
    case 16: return moe_launch_n<16, FMT, EPI>(map, a, ctas, s);
    case 32: return moe_launch_n<32, FMT, EPI>(map, a, ctas, s);
    case 64: return moe_launch_n<64, FMT, EPI>(map, a, ctas, s);
    case 128: return moe_launch_n<128, FMT, EPI>(map, a, ctas, s);
    default: return -1;
  }
}

int launch_moe_gemm_tc(int fmt, int epi, const void* w, int rows, int K, const void* xs,
                       int xs_stride, int xs_rows, int tok_tile, const void* tiles,
                       const int* n_tiles, int max_tiles, const float* bias, int bias_stride,
                       void* h, int h_stride, int act_kind, float alpha, float limit,
                       const unsigned long long* out_ptrs, int n_out, int out_stride,
                       const int32_t* ret, int num_sms, int* status, cudaStream_t s,
                       int* sig_ctl, const unsigned long long* sig_bases, long long sig_flag_off,
                       int sig_world, int sig_rank) {
  if (K < 64) return -1;  // every item's first unit feeds all (<= 4) sub-accumulators
  if (fmt == kMoeFmtQ4K && K % 256) return -1;
  if (fmt == kMoeFmtMX && K % 64) return -1;  // TMA boxes + the bf16 pair layout
  if (epi == kMoeEpiSwiglu && (rows % 128)) return -1;  // 64 features (gate + up) per tile
  if (n_out > 8) return -1;
  if ((xs_stride % 8) || (reinterpret_cast<uintptr_t>(xs) & 15)) return -5;
  const int rows_pad = (rows + 127) / 128 * 128;
  const int n_units = (K + 255) / 256;
  const int last_k = K - (n_units - 1) * 256;
  MoeGemmArgs a{};
  a.w = (const uint8_t*)w;
  a.w_expert_bytes = moe_packed_bytes(fmt, rows, K);
  a.row_tiles = rows_pad / 128;
  a.w_tile_bytes = a.w_expert_bytes / a.row_tiles;
  a.w_last_bytes = fmt == kMoeFmtQ4K ? 128 * kQ4kRowBytes : 128 * (8 + 16 * (last_k / 32));
  a.rows_valid = epi == kMoeEpiSwiglu ? rows / 2 : rows;
  a.n_units = n_units;
  a.last_k = last_k;
  a.tiles = (const int4*)tiles;
  a.n_tiles = n_tiles;
  a.bias = bias;
  a.bias_stride = bias_stride;
  a.h = h;
  a.h_stride = h_stride;
  a.act_kind = act_kind;
  a.alpha = alpha;
  a.limit = limit;
  for (int i = 0; i < n_out; ++i) a.out_ptrs[i] = out_ptrs[i];
  a.out_stride = out_stride;
  a.ret = ret;
  a.status = status;
  a.sig_ctl = sig_ctl;
  if (sig_ctl) {
    if (sig_world > 8) return -1;
    for (int i = 0; i < sig_world; ++i) a.sig_bases[i] = sig_bases[i];
    a.sig_flag_off = sig_flag_off;
    a.sig_world = sig_world;
    a.sig_rank = sig_rank;
  }
  CUtensorMap map;
  if (make_tmap_2d_16bit(&map, xs, xs_rows, K, xs_stride, tok_tile, 64, 128) != 0) return -2;
  const long long items = (long long)max_tiles * a.row_tiles;
  int ctas = (int)(items < num_sms ? items : num_sms);
  if (ctas <= 0) {
    if (!sig_ctl) return 0;
    ctas = 1;  // the peers wait for the completion signal even when there is no work
  }
  if (fmt == kMoeFmtQ4K)
    return epi == kMoeEpiSwiglu ? moe_launch_fmt<kMoeFmtQ4K, kMoeEpiSwiglu>(tok_tile, map, a, ctas, s)
                                : moe_launch_fmt<kMoeFmtQ4K, kMoeEpiStore>(tok_tile, map, a, ctas, s);
  return epi == kMoeEpiSwiglu ? moe_launch_fmt<kMoeFmtMX, kMoeEpiSwiglu>(tok_tile, map, a, ctas, s)
                              : moe_launch_fmt<kMoeFmtMX, kMoeEpiStore>(tok_tile, map, a, ctas, s);
}

// Small batches: a cluster of 8 CTAs per token splits the row; the RMSNorm's
// sum of squares is reduced through distributed shared memory.
__global__ void __launch_bounds__(256) moe_combine_cluster_kernel(
    const float* __restrict__ rows, int row_stride, const float* __restrict__ wts, int k,
    GemmOut sh, int has_sh, GemmOut shg, int has_shg, float* __restrict__ residual, int H,
    const float* __restrict__ norm_w, __half* __restrict__ out, int out_stride, float eps) {
  pdl_trigger();  // dependents (the next GEMM) may launch and prefetch weights
  pdl_wait();     // what earlier kernels wrote is complete and visible
  cg::cluster_group cluster = cg::this_cluster();
  __shared__ float part;
  __shared__ float red[32];
  extern __shared__ float cslice[];
  const int cr = (int)cluster.block_rank(), cn = (int)cluster.num_blocks();
  const int t = blockIdx.x / cn;
  const int per = (H + cn - 1) / cn;
  const int lo = cr * per, hi = min(H, lo + per);
  float gate = 1.f;
  if (has_shg) gate = 1.f / (1.f + __expf(-shg.get(t, 0)));
  float ss = 0.f;
  for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    float v = 0.f;
    for (int j = 0; j < k; ++j) v += wts[t * k + j] * rows[(size_t)(t * k + j) * row_stride + i];
    if (has_sh) v += gate * sh.get(t, i);
    const float r = residual[(size_t)t * H + i] + v;
    residual[(size_t)t * H + i] = r;
    cslice[i - lo] = r;
    ss += r * r;
  }
  ss = block_sum(ss, red);
  if (threadIdx.x == 0) part = ss;
  cluster.sync();
  float tot = 0.f;
  for (int r = 0; r < cn; ++r) tot += *cluster.map_shared_rank(&part, r);
  cluster.sync();
  if (out == nullptr) return;
  const float inv = rsqrtf(tot / H + eps);
  for (int i = lo + threadIdx.x; i < hi; i += blockDim.x)
    out[(size_t)t * out_stride + i] = __float2half_rn(cslice[i - lo] * inv * norm_w[i]);
}

int launch_moe_combine(const float* rows, int row_stride, const float* wts, int k,
                       const GemmOut* sh, const GemmOut* shg, float* residual, int T, int H,
                       const float* norm_w, __half* out, int out_stride, float eps,
                       cudaStream_t s) {
  if (T <= 0) return 0;
  GemmOut z{};
  if (T < 64) {
    constexpr int kC = 8;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(T * kC);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = (size_t)((H + kC - 1) / kC) * sizeof(float);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kC;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, moe_combine_cluster_kernel, rows, row_stride, wts, k,
                       sh ? *sh : z, (int)(sh != nullptr), shg ? *shg : z, (int)(shg != nullptr),
                       residual, H, norm_w, out, out_stride ? out_stride : H, eps);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : -2;
  }
  const size_t smem = (size_t)H * 4;
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(moe_combine_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
  moe_combine_kernel<<<T, 512, smem, s>>>(rows, row_stride, wts, k, sh ? *sh : z, sh != nullptr,
                                          shg ? *shg : z, shg != nullptr, residual, H, norm_w,
                                          out, out_stride ? out_stride : H, eps);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -2;
}

int launch_moe_localize(int32_t* ids, float* wts, int* counts, int P, int E, int e0, int n_loc,
                        cudaStream_t s) {
  if (E > 1024 || e0 < 0 || n_loc <= 0 || e0 + n_loc > E) return -1;
  moe_localize_kernel<<<1, 1024, 0, s>>>(ids, wts, counts, P, E, e0, n_loc);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -2;
}

int launch_moe_combine_tp(const float* rows, int row_stride, const float* wts, int k,
                          const GemmOut* sh, const GemmOut* shg, int T, int H, int W,
                          const unsigned long long* dst, int* ctl, const unsigned long long* bases,
                          long long flag_off, int rank, cudaStream_t s, int to_all) {
  if (T <= 0) return 0;
  if (W < 1 || W > 8 || H % W) return -1;
  GemmOut z{};
  EpPeers d{}, b{};
  for (int i = 0; i < W; ++i) {
    d.base[i] = dst[i];
    b.base[i] = bases[i];
  }
  moe_combine_tp_kernel<<<T, 256, 0, s>>>(rows, row_stride, wts, k, sh ? *sh : z,
                                          (int)(sh != nullptr), shg ? *shg : z,
                                          (int)(shg != nullptr), H, W, d, ctl, b, flag_off, rank,
                                          to_all);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -2;
}
