// Quantized x fp16 GEMV for decode at 1..2 tokens, on the CUDA cores.
//
//   out[t][r] = sum_k W[r][k] * X[t][k],   W: Q4_K / Q6_K / Q8_0 (repacked, as
//   qgemm_tc.cu; the per-format row math is in qfmt.cuh), X: fp16 [T, K]
//
// At a handful of tokens the GEMM is a weight stream.  On the tensor cores a
// 128 x N x 16 tcgen05.mma costs the same ~48 clocks for every N <= 64 and
// the hand-offs around it stretch that further, so the swap-AB kernel tops
// out near a third of HBM bandwidth there; this kernel works on the CUDA
// cores instead.  (Reference: the mmvq dp4a path for <= 8 rows, candle
// quantized/cuda.rs:291.)
//
// Layout and decomposition (shared with the tensor-core kernel, so the
// stream-K partial format read by every epilogue -- gemm_out.cuh -- is the
// same): a unit is (128-row tile, 256-K superblock); CTAs take contiguous
// unit ranges; the partial of each tile segment goes to slot (tile + cta).
// Inside a CTA, warp w owns rows [32w, 32w+32) of every unit: it streams its
// quarter of the unit (32 repacked rows, 2 stages) and the unit's activations (T x 512 B,
// 2 stages) into its own shared memory with bulk copies, so no warp ever
// waits on another.  One lane = one weight row.
//
// Q4_K (the common case) runs on integer dot products: each warp quantizes
// the unit's activations to int8 (one scale per 32 values, as llama.cpp's
// q8_1 activations for its mmvq kernels), then per 32-bit word of codes (8
// weights) two masks split the nibbles into int8x4 words and two dp4a
// accumulate them; the sub-block scale and min are applied once per 32
// weights in fp32 (qfmt.cuh FmtQ4K::gemv_i8).  That is about 5 issue slots
// per 8 weights instead of 13 for fp16 dequantization, so the weight stream
// is no longer issue-bound; the activation rounding adds ~0.5 % relative
// error.  Q8_0 does the same with its byte codes (activations in plain K
// order), Q6_K with its 6-bit codes rebuilt as bytes.  SWARMLLM_GEMV_I8=0
// selects the fp16 paths (F::gemv); the mixed Q4_K|Q6_K GEMV always takes them.
#include "kernels.h"

#include <cstdlib>
#include <type_traits>

#include "common.cuh"
#include "ep_common.cuh"
#include "gemm_out.cuh"
#include "qfmt.cuh"
#include "tc_utils.cuh"

namespace swarm {
using namespace tc;

constexpr int kGvWarps = 4;                          // one per 32-row quarter of a tile
constexpr int kGvWStages = 2;                        // code stages per warp
constexpr int kGvXStages = 2;                        // activation stages per warp
// mbarriers of all warps, ahead of the stage buffers
constexpr int kGvBarBytes = 256;
static_assert(kGvWarps * (kGvWStages + kGvXStages) * 8 <= kGvBarBytes, "barrier area too small");

template <class F, class FB, int T, bool I8 = false>
struct GvCfg {
  static constexpr int ROW_MAX = F::ROW_BYTES > FB::ROW_BYTES ? F::ROW_BYTES : FB::ROW_BYTES;
  static constexpr int QUARTER = 32 * ROW_MAX;              // one warp's rows of a unit
  static constexpr int X_STAGE = T * 512;                   // T x 256 fp16
  static constexpr int XQ_BYTES = I8 ? T * (256 + 64) : 0;  // int8 x + (dx, sum) per 32
  static constexpr int WARP_BYTES = kGvWStages * QUARTER + kGvXStages * X_STAGE + XQ_BYTES;
  static constexpr int SMEM = kGvBarBytes + kGvWarps * WARP_BYTES;
  static_assert(WARP_BYTES % 16 == 0 &&
                    qgemv_ctas_per_sm(ROW_MAX == F::ROW_BYTES ? F::ID : FB::ID, T) *
                            (SMEM + 1024) <= 228 * 1024,
                "stage layout");
};

struct GemvArgs {
  const uint8_t* w;
  const uint8_t* w_b;  // row tiles >= split_tile: second format's tensor (mixed-format GEMV)
  int split_tile;
  const __half* x;
  int x_stride;   // elements
  int rows, K;
  int ksb;
  long total_units;
  int upc;
  float* ws;
  int* status;
  int n_peers;
  unsigned long long peer_ws[8];
  int owner_tiles;  // > 0: row tile rt goes only to rank rt / owner_tiles (reduce-scatter)
  int* sig_ctl;
  unsigned long long sig_bases[8];
  long long sig_flag_off;
  int sig_rank;
};

// One unit of one warp: codes from the stage into registers (the stage is then
// refilled), wait for the unit's activations, accumulate the dot products.
template <class F, int T, bool I8, class IssueW>
SW_DEVICE bool gemv_unit(const uint8_t* stage, uint64_t* xb, const uint8_t* xstage, uint8_t* xq,
                         int i, float (&acc)[T], int w_next, int n, IssueW& issue_w, int* status,
                         int warp, int lane) {
  typename F::Regs r;
  F::load(reinterpret_cast<const uint4*>(stage + lane * F::ROW_BYTES), r);
  __syncwarp();
  if (lane == 0 && w_next < n) issue_w();
  F::gemv_prep(r);
  if (!mbar_wait_warp(xb, (i / kGvXStages) & 1, status, 42, i, warp)) return false;
  mbar_try_wait(smem_u32(xb), (i / kGvXStages) & 1);
  if constexpr (I8) {
    uint2* xq8 = reinterpret_cast<uint2*>(xq);
    float2* xs2 = reinterpret_cast<float2*>(xq + T * 256);
    quantize_x8<T, F::X8_NATURAL>(reinterpret_cast<const uint4*>(xstage), xq8, xs2, lane);
    __syncwarp();
    F::template gemv_i8<T>(r, xq8, xs2, acc);
  } else {
    F::template gemv<T>(r, reinterpret_cast<const uint4*>(xstage), acc, lane);
  }
  return true;
}

template <class F, class FB, int T, bool I8>
__global__ void __launch_bounds__(kGvWarps * 32)
    qgemv_q4k_kernel(const __grid_constant__ GemvArgs a) {
  using C = GvCfg<F, FB, T, I8>;
  constexpr bool kMixed = !std::is_same<F, FB>::value;
  extern __shared__ __align__(128) uint8_t gv_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint64_t* wfull = reinterpret_cast<uint64_t*>(gv_smem) + warp * (kGvWStages + kGvXStages);
  uint64_t* xfull = wfull + kGvWStages;
  uint8_t* wst = gv_smem + kGvBarBytes + warp * C::WARP_BYTES;
  uint8_t* xst = wst + kGvWStages * C::QUARTER;
  uint8_t* xq = xst + kGvXStages * C::X_STAGE;   // int8 activations (I8 only)

  const long u0 = (long)blockIdx.x * a.upc;
  const long u1 = min(a.total_units, u0 + a.upc);
  const int n = (int)max(0L, u1 - u0);
  pdl_trigger();   // the next kernel (an epilogue) may launch now; it waits for this grid

  if (lane == 0) {
    for (int s = 0; s < kGvWStages + kGvXStages; ++s) mbar_init(&wfull[s], 1);
    fence_barrier_init();
  }
  __syncwarp();

  // bulk copies of unit i: this warp's 32 rows of codes, and the activations.
  // A code stage is refilled as soon as its codes are in registers, an
  // activation stage once the unit's dot products are done.  Units are walked
  // with (tile, superblock) cursors: one division per CTA, none per unit.
  const int rt0 = (int)(u0 / a.ksb), sb0 = (int)(u0 - (long)rt0 * a.ksb);
  int w_next = 0, x_next = 0, x_sb = sb0;   // lane 0's copy cursors
  int w_rt = rt0, w_sb = sb0;
  auto issue_w = [&]() {                    // this warp's 32 rows of unit w_next
    uint64_t* bar = &wfull[w_next % kGvWStages];
    const uint8_t* src;
    int bytes;
    if (kMixed && w_rt >= a.split_tile) {
      bytes = 32 * FB::ROW_BYTES;
      src = a.w_b + (((size_t)(w_rt - a.split_tile) * a.ksb + w_sb) * 128 + warp * 32) *
                        FB::ROW_BYTES;
    } else {
      bytes = 32 * F::ROW_BYTES;
      src = a.w + (((size_t)w_rt * a.ksb + w_sb) * 128 + warp * 32) * F::ROW_BYTES;
    }
    mbar_arrive_expect_tx(bar, bytes);
    bulk_load(wst + (w_next % kGvWStages) * C::QUARTER, src, bytes, bar);
    ++w_next;
    if (++w_sb == a.ksb) {
      w_sb = 0;
      ++w_rt;
    }
  };
  auto issue_x = [&]() {
    uint64_t* bar = &xfull[x_next % kGvXStages];
    mbar_arrive_expect_tx(bar, C::X_STAGE);
#pragma unroll
    for (int t = 0; t < T; ++t)
      bulk_load(xst + (x_next % kGvXStages) * C::X_STAGE + t * 512,
                a.x + (size_t)t * a.x_stride + (size_t)x_sb * 256, 512, bar);
    ++x_next;
    if (++x_sb == a.ksb) x_sb = 0;
  };
  if (lane == 0) {
    while (w_next < min(n, kGvWStages)) issue_w();   // weights: independent of the previous kernel
    pdl_wait();                                      // activations and results: after it
    while (x_next < min(n, kGvXStages)) issue_x();
  }

  float acc[T];
#pragma unroll
  for (int t = 0; t < T; ++t) acc[t] = 0.f;

  bool ok = true;
  int rt = rt0, sb = sb0;
  for (int i = 0; i < n; ++i) {
    uint64_t* wb = &wfull[i % kGvWStages];
    if (!(ok = mbar_wait_warp(wb, (i / kGvWStages) & 1, a.status, 41, i, warp))) break;
    mbar_try_wait(smem_u32(wb), (i / kGvWStages) & 1);   // every lane acquires the bytes
    const uint8_t* stage = wst + (i % kGvWStages) * C::QUARTER;
    uint64_t* xb = &xfull[i % kGvXStages];
    if (kMixed && rt >= a.split_tile)
      ok = gemv_unit<FB, T, false>(stage, xb, xst + (i % kGvXStages) * C::X_STAGE, xq, i, acc,
                                   w_next, n,
                            issue_w, a.status, warp, lane);
    else
      ok = gemv_unit<F, T, I8>(stage, xb, xst + (i % kGvXStages) * C::X_STAGE, xq, i, acc,
                               w_next, n,
                           issue_w, a.status, warp, lane);
    if (!ok) break;

    __syncwarp();   // every lane is done with this activation stage
    if (lane == 0 && x_next < n) issue_x();
    if (i == n - 1 || sb == a.ksb - 1) {
      // tile segment done: partial into slot (tile + cta), token rows 0..T-1 of 16
      const size_t off = ((size_t)(rt + blockIdx.x) * 16) * 128 + warp * 32 + lane;
      if (a.n_peers == 0) {
#pragma unroll
        for (int t = 0; t < T; ++t) a.ws[off + (size_t)t * 128] = acc[t];
      } else {
        const int o0 = a.owner_tiles > 0 ? rt / a.owner_tiles : 0;
        const int o1 = a.owner_tiles > 0 ? o0 + 1 : a.n_peers;
        for (int o = o0; o < o1; ++o) {
          float* dst = reinterpret_cast<float*>(a.peer_ws[o]) + off;
#pragma unroll
          for (int t = 0; t < T; ++t) dst[(size_t)t * 128] = acc[t];
        }
      }
#pragma unroll
      for (int t = 0; t < T; ++t) acc[t] = 0.f;
    }
    if (++sb == a.ksb) {
      sb = 0;
      ++rt;
    }
  }
  if (!ok && lane == 0) {  // let this warp's copies still in flight land before exiting
    for (int i = max(0, w_next - kGvWStages); i < w_next; ++i)
      mbar_wait(&wfull[i % kGvWStages], (i / kGvWStages) & 1, nullptr, 0);
    for (int i = max(0, x_next - kGvXStages); i < x_next; ++i)
      mbar_wait(&xfull[i % kGvXStages], (i / kGvXStages) & 1, nullptr, 0);
  }
  __syncwarp();
  if (a.sig_ctl != nullptr)   // all threads of every CTA (it syncs the CTA itself)
    ep_grid_done_signal(a.sig_ctl, a.sig_bases, a.sig_flag_off, a.n_peers, a.sig_rank);
}

// The plan assumes qgemv_ctas_per_sm(fmt, T) CTAs resident per SM (one wave);
// ask for the full shared-memory carveout so they fit.
template <class F, class FB, int T, bool I8>
static int setup_t() {
  // Function attributes apply to the current device: set them once per device.
  static unsigned long long done = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -3;
  const unsigned long long bit = 1ull << dev;
  if (__atomic_load_n(&done, __ATOMIC_ACQUIRE) & bit) return 1;
  if (cudaFuncSetAttribute(qgemv_q4k_kernel<F, FB, T, I8>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                           GvCfg<F, FB, T, I8>::SMEM) != cudaSuccess ||
      cudaFuncSetAttribute(qgemv_q4k_kernel<F, FB, T, I8>,
                           cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess)
    return -3;
  __atomic_fetch_or(&done, bit, __ATOMIC_RELEASE);
  return 1;
}

template <class F, int T>
static int occupancy_t() {
  constexpr bool I8 = F::HAS_I8;
  if (setup_t<F, F, T, I8>() != 1) return -1;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, qgemv_q4k_kernel<F, F, T, I8>,
                                                    kGvWarps * 32,
                                                    GvCfg<F, F, T, I8>::SMEM) != cudaSuccess)
    return -1;
  return n;
}

template <class F, class FB, int T, bool I8>
static int launch_t(const GemvArgs& a, int ctas, cudaStream_t s) {
  if (setup_t<F, FB, T, I8>() != 1) return -3;
  if (launch_pdl(qgemv_q4k_kernel<F, FB, T, I8>, dim3(ctas), dim3(kGvWarps * 32),
                 GvCfg<F, FB, T, I8>::SMEM, s, a) != cudaSuccess)
    return -4;
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}

// Q4_K, Q6_K and Q8_0 (unmixed) take the integer-dot variant unless SWARMLLM_GEMV_I8=0.
static const bool g_gemv_i8 = [] {
  const char* v = getenv("SWARMLLM_GEMV_I8");
  return v ? atoi(v) != 0 : true;
}();

template <class F, class FB = F>
static int launch_f(const GemvArgs& a, int T, int ctas, cudaStream_t s) {
  if constexpr (F::HAS_I8 && std::is_same<F, FB>::value) {
    if (g_gemv_i8)
      return T == 1 ? launch_t<F, FB, 1, true>(a, ctas, s) : launch_t<F, FB, 2, true>(a, ctas, s);
  }
  return T == 1 ? launch_t<F, FB, 1, false>(a, ctas, s) : launch_t<F, FB, 2, false>(a, ctas, s);
}

}  // namespace swarm

using namespace swarm;

int q4k_gemv_occupancy(int T, int fmt) {
  if (T != 1 && T != 2) return 0;
  switch (fmt) {
    case kFmtQ4K: return T == 1 ? occupancy_t<FmtQ4K, 1>() : occupancy_t<FmtQ4K, 2>();
    case kFmtQ6K: return T == 1 ? occupancy_t<FmtQ6K, 1>() : occupancy_t<FmtQ6K, 2>();
    case kFmtQ8_0: return T == 1 ? occupancy_t<FmtQ80, 1>() : occupancy_t<FmtQ80, 2>();
    default: return 0;
  }
}

int launch_qgemv_q4k(const void* w_packed, int rows, int K, const __half* x, int x_stride, int T,
                     float* ws, int ksb, long total_units, int upc, int ctas, int* status,
                     const unsigned long long* peer_ws, int n_peers, int* sig_ctl,
                     const unsigned long long* sig_bases, long long sig_flag_off, int sig_rank,
                     cudaStream_t s, int owner_tiles, int fmt, const void* w_b, int fmt_b,
                     int split_tile) {
  if (T < 1 || T > kQGemvMaxT || fmt < 0 || fmt >= kNumQFmts) return -1;
  const bool mixed = w_b != nullptr && fmt_b >= 0 && fmt_b != fmt;
  if (mixed && !(fmt == kFmtQ4K && fmt_b == kFmtQ6K)) return -1;
  if ((x_stride % 8) != 0 || (reinterpret_cast<uintptr_t>(x) & 15) != 0 ||
      (reinterpret_cast<uintptr_t>(w_packed) & 15) != 0)
    return -5;
  GemvArgs a{};
  a.w = static_cast<const uint8_t*>(w_packed);
  a.w_b = mixed ? static_cast<const uint8_t*>(w_b) : nullptr;
  a.split_tile = mixed ? split_tile : 0;
  a.x = x;
  a.x_stride = x_stride;
  a.rows = rows;
  a.K = K;
  a.ksb = ksb;
  a.total_units = total_units;
  a.upc = upc;
  a.ws = ws;
  a.status = status;
  a.n_peers = 0;
  a.sig_ctl = nullptr;
  if (n_peers > 0) {
    if (n_peers > 8 || !peer_ws || !sig_ctl || !sig_bases) return -7;
    a.n_peers = n_peers;
    for (int i = 0; i < n_peers; ++i) {
      a.peer_ws[i] = peer_ws[i];
      a.sig_bases[i] = sig_bases[i];
    }
    a.sig_ctl = sig_ctl;
    a.sig_flag_off = sig_flag_off;
    a.sig_rank = sig_rank;
    a.owner_tiles = owner_tiles;
    if (owner_tiles > 0 && (rows / 128) > owner_tiles * n_peers) return -7;
  }
  if (mixed) return launch_f<FmtQ4K, FmtQ6K>(a, T, ctas, s);
  switch (fmt) {
    case kFmtQ4K: return launch_f<FmtQ4K>(a, T, ctas, s);
    case kFmtQ6K: return launch_f<FmtQ6K>(a, T, ctas, s);
    default: return launch_f<FmtQ80>(a, T, ctas, s);
  }
}
