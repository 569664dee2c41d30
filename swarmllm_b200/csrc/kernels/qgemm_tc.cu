// Quantized x fp16 GEMM on the 5th-generation tensor cores (tcgen05 / TMEM / TMA).
//
//   out[t][r] = sum_k W[r][k] * X[t][k],   W: Q4_K, Q6_K or Q8_0 (repacked), X: fp16 [T, K]
//
// The kernel is written once over a weight format (qfmt.cuh: repacked row
// size, register dequantizer); the description below uses Q4_K.
//
// One kernel serves decode (T = 1..256 tokens, weight-streaming, bound by HBM)
// and prefill (T up to thousands, tensor-bound).  It replaces the reference's
// three quantized paths (candle mmvq dp4a for <= 8 rows, llama.cpp MMQ
// mma.sync int8, and dequantize-to-f16 + cuBLAS for >= 64 rows:
// vendor/candle/candle-core/src/quantized/cuda.rs:291,519,1005).
//
// Design (swap-AB weight streaming):
//  * The MMA's M dimension is 128 weight rows; N is the token tile (16..256).
//  * Weights are repacked once at load time (launch_q4k_repack) into
//    [row_tile][superblock][128 rows][144 B]: 128 B of 4-bit codes whose
//    nibbles are ordered so that one LOP3 yields two consecutive K values as
//    an fp16 pair (1024 + q) -- then an exact subtract and one HFMA2 apply the
//    6-bit sub-block scale and min -- followed by the 16 B (d, dmin, scales).
//    A 128-row x 256-K chunk is one contiguous 18 KB bulk copy.
//  * Dequantizer warps (one thread per weight row) write the fp16 weights
//    straight into TMEM and the MMA reads its A operand from TMEM
//    (tcgen05.mma ... [a_tmem]); shared memory only carries the raw 4.5-bit
//    codes and the activations, so it is not the bottleneck at decode.
//  * Activations arrive by TMA (128 B swizzle, K-major canonical layout) into
//    their own ring of up to 8 unit tiles, loaded well ahead of the MMAs; the
//    fp32 accumulator lives in TMEM columns [0, N).
//  * Persistent, stream-K balanced: the (row_tile, token_tile, superblock)
//    units are split evenly over the CTAs; each CTA writes one fp32 partial
//    per tile it touched into workspace slot (tile + cta); epilogue kernels
//    sum the slots while reading (gemm_out.cuh).
//
// Warp roles: warp 0 = bulk/TMA producer, warp 1 = TMEM owner + MMA issuer,
// warps 2.. = 3 (token tile <= 128) or 2 dequantizer warpgroups taking units
// round-robin; warpgroup 0 also drains the accumulator at the end of every
// tile segment.
#include "kernels.h"

#include <cstdlib>
#include <type_traits>
#include "gemm_out.cuh"
#include "qfmt.cuh"
#include "tc_utils.cuh"
#include "ep_common.cuh"

namespace swarm {
using namespace tc;

constexpr int kTmemCols = 512;

// Per token-tile configuration.
template <class F, class FB, int N>
struct QCfg {
  // Dequantizer warpgroups take units round-robin; each owns one "unit stage"
  // of 128 TMEM columns (A for K = 256 fp16), released by MMA commits.  The W
  // stage counts are multiples of DQ, so every W stage is re-used by the
  // warpgroup that used it last and no parity wait can run two phases ahead.
  static constexpr int DQ = N <= 64 ? 3 : 2;
  static constexpr int U = DQ;                           // unit stages in flight
  // Hand-offs per unit between the dequantizers and the MMA issuer: 2 = per
  // K half (64 columns), each dequantized into registers before its TMEM
  // half is free, so the first half's MMAs overlap the second half's
  // dequantization; 1 = whole units, dequantized after the wait.
// Timing experiments only (results are wrong): 1 = dequantizers skip the
// TMEM writes, 2 = the MMA issuer skips the MMAs (commits still flow).
#ifndef SWARMLLM_QGEMM_EXPERIMENT
#define SWARMLLM_QGEMM_EXPERIMENT 0
#endif
#ifndef SWARMLLM_QGEMM_HALVES
#define SWARMLLM_QGEMM_HALVES 1
#endif
// Activation ring depth: 0 = tied to the TMEM A stages (one MMA commit per
// unit releases both), else the deepest ring that fits (its own commit).
#ifndef SWARMLLM_QGEMM_XRING
#define SWARMLLM_QGEMM_XRING 0
#endif
  static constexpr int HALVES = SWARMLLM_QGEMM_HALVES;
  static constexpr int THREADS = 96 + 128 * DQ;          // W producer, MMA, X producer, DQ WGs
  static constexpr int FIRST_DQ_WARP = 3;
  static constexpr int A_COL = kTmemCols - 128 * U;      // accumulators use [0, NACC * N)
  // Independent accumulators the 16 MMAs of a unit rotate over.  At decode
  // sizes a 128 x N x 16 MMA is short, and MMAs that accumulate into the same
  // TMEM columns wait for each other; rotating over NACC accumulators keeps
  // NACC of them in flight.  The drain adds the accumulators.
  static constexpr int NACC = (A_COL / N) >= 4 ? 4 : ((A_COL / N) >= 2 ? 2 : 1);
  static constexpr int X_UNIT_BYTES = N * 512;           // N rows x 256 K fp16 (4 swizzle atoms)
  // A stage holds one unit of either format (FB: the row tiles from split_tile on).
  static constexpr int ROW_MAX = F::ROW_BYTES > FB::ROW_BYTES ? F::ROW_BYTES : FB::ROW_BYTES;
  static constexpr int W_STAGE = 128 * ROW_MAX;          // 18 KB for Q4_K
  static_assert(A_COL >= NACC * N, "TMEM budget");
  static constexpr int BAR_BYTES = 512;
  // Activation tiles: by default one per TMEM A stage, released by the same
  // MMA commit (each tcgen05.commit costs the pipe a drain; see the MMA
  // probe).  With SWARMLLM_QGEMM_XRING they get their own ring, X_ST units
  // deep, released by a commit of their own.
  // Two W stages per warpgroup unless that costs X stages below 4.
  static constexpr int x_room(int w_st) {
    return (227 * 1024 - 1024 - BAR_BYTES - w_st * W_STAGE) / X_UNIT_BYTES;
  }
  static constexpr int W_ST =
      x_room(2 * DQ) >= (x_room(DQ) < 4 ? x_room(DQ) : 4) ? 2 * DQ : DQ;
  static constexpr bool X_TIED = SWARMLLM_QGEMM_XRING == 0;
  static constexpr int X_ST = X_TIED ? U : (x_room(W_ST) < 8 ? x_room(W_ST) : 8);
  static_assert(X_ST >= 2, "activation ring");
  static constexpr int X_BYTES = X_ST * X_UNIT_BYTES;
  static constexpr int W_BYTES = W_ST * W_STAGE;
  static constexpr int SMEM = 1024 + X_BYTES + W_BYTES + BAR_BYTES;
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  static_assert((2 * W_ST + 2 * U * HALVES + 2 * X_ST + 3) * 8 + 4 <= BAR_BYTES, "barriers");
};

struct QGemmArgs {
  const uint8_t* w;
  const uint8_t* w_b;  // row tiles >= split_tile: second format's tensor (mixed-format GEMM)
  int split_tile;
  int rows, K, T;
  int n_tok_tiles, ksb;
  long total_units;
  int upc;
  float* ws;
  int* status;
  unsigned long long* trace;  // debug: per-unit event timestamps of CTA 0 (null = off)
  // Tensor parallelism: when n_peers > 0 the partial tiles go to every rank's
  // receive buffer (peer_ws[o], over NVLink) instead of `ws`, and the CTA that
  // finishes last raises flag word sig_bases[o] + sig_flag_off + 4 * sig_rank.
  int n_peers;
  unsigned long long peer_ws[8];
  int owner_tiles;  // > 0: row tile rt goes only to rank rt / owner_tiles (reduce-scatter)
  int* sig_ctl;
  unsigned long long sig_bases[8];
  long long sig_flag_off;
  int sig_rank;
};

// Debug timeline of CTA 0 (see qgemm_set_trace): trace[unit*8 + event] = %globaltimer.
// Compiled in only with -DSWARMLLM_KERNEL_TRACE (setup.py: SWARMLLM_KERNEL_TRACE=1).
#ifdef SWARMLLM_KERNEL_TRACE
#define QTRACE(tr, unit, ev)                                                           \
  do {                                                                                 \
    if ((tr) != nullptr && blockIdx.x == 0 && (unit) < 512) (tr)[(unit) * 8 + (ev)] = \
        globaltimer();                                                                 \
  } while (0)
#else
#define QTRACE(tr, unit, ev) \
  do {                       \
  } while (0)
#endif

// One dequantizer warp's part of a unit: stage -> registers (freeing the
// stage), then the unit's TMEM A stage in H hand-offs (H = 2: one per K half
// of 64 columns).  With H = 2 each half is dequantized into registers BEFORE
// waiting for the MMAs that last read that half of the stage, so the wait is
// followed only by the TMEM stores: the stage turns around in the time of the
// stores, not of the dequantization.
template <class F, int H>
SW_DEVICE bool dq_unit_fmt(const uint8_t* stage, int row, uint64_t* w_empty, uint64_t* empty_h,
                           uint64_t* ready_h, uint32_t empty_parity, uint32_t taddr, int* status,
                           int i, int lane) {
  typename F::Regs r;
  F::load(reinterpret_cast<const uint4*>(stage + row * F::ROW_BYTES), r);
  __syncwarp();
  if (lane == 0) mbar_arrive(w_empty);
  F::prep(r);
#pragma unroll
  for (int h = 0; h < H; ++h) {
    if constexpr (H == 2) {
      uint32_t cols[64];
      dq_half_regs<F>(r, h, cols);
      if (!mbar_wait_warp(&empty_h[h], empty_parity, status, 32, i, h)) return false;
      tc_fence_after();
#if SWARMLLM_QGEMM_EXPERIMENT != 1
      store_half(taddr, h, cols);
#endif
    } else {
      if (!mbar_wait_warp(&empty_h[h], empty_parity, status, 32, i, h)) return false;
      tc_fence_after();
#if SWARMLLM_QGEMM_EXPERIMENT != 1
      dq_unit_store<F>(r, taddr);
#endif
    }
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&ready_h[h]);
  }
  return true;
}

template <class F, class FB, int N>
__global__ void __launch_bounds__(QCfg<F, FB, N>::THREADS, 1)
    qgemm_q4k_tc_kernel(const __grid_constant__ CUtensorMap x_map, QGemmArgs a) {
  using C = QCfg<F, FB, N>;
  constexpr bool kMixed = !std::is_same<F, FB>::value;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* x_smem = smem;
  uint8_t* w_smem = smem + C::X_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(w_smem + C::W_BYTES);
  uint64_t* w_full = bars;                 // W stage loaded (tx)
  uint64_t* w_empty = w_full + C::W_ST;    // W stage read by its warpgroup (4 warps)
  // Per unit stage s and hand-off h (index s * HALVES + h):
  uint64_t* ready = w_empty + C::W_ST;     // A part in TMEM (4 warps)
  uint64_t* empty = ready + C::HALVES * C::U;   // A part consumed by the MMAs (commit)
  uint64_t* x_full = empty + C::HALVES * C::U;  // activation stage loaded (tx)
  uint64_t* x_empty = x_full + C::X_ST;         // activation stage consumed (commit)
  uint64_t* d_full = x_empty + C::X_ST;
  uint64_t* d_empty = d_full + 1;
  uint64_t* done_bar = d_empty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long u0 = (long)blockIdx.x * a.upc;
  const long u1 = min(a.total_units, u0 + a.upc);
  const int n_units = (int)max(0L, u1 - u0);
  // the next kernel (an epilogue) may launch now; it waits for this grid
  pdl_trigger();

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::W_ST; ++i) { mbar_init(&w_full[i], 1); mbar_init(&w_empty[i], 4); }
    for (int i = 0; i < C::U * C::HALVES; ++i) {
      mbar_init(&ready[i], 4);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < C::X_ST; ++i) {
      mbar_init(&x_full[i], 1);
      mbar_init(&x_empty[i], 1);
    }
    mbar_init(d_full, 1);
    mbar_init(d_empty, 4);
    mbar_init(done_bar, 1);
    fence_barrier_init();
    prefetch_tensormap(&x_map);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
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
      int tile = (int)(u0 / a.ksb), sb = (int)(u0 - (long)tile * a.ksb);
      for (int i = 0; i < n_units && ok; ++i, (++sb == a.ksb) ? (sb = 0, ++tile) : 0) {
        const int rt = tile / a.n_tok_tiles;
        const int wsi = i % C::W_ST;
        if (!(ok = mbar_wait(&w_empty[wsi], ((i / C::W_ST) & 1) ^ 1, a.status, 11, i, 0))) break;
        QTRACE(a.trace, i, 0);
        const uint8_t* wsrc;
        int bytes;
        if (kMixed && rt >= a.split_tile) {
          bytes = 128 * FB::ROW_BYTES;
          wsrc = a.w_b + ((size_t)(rt - a.split_tile) * a.ksb + sb) * bytes;
        } else {
          bytes = 128 * F::ROW_BYTES;
          wsrc = a.w + ((size_t)rt * a.ksb + sb) * bytes;
        }
        mbar_arrive_expect_tx(&w_full[wsi], bytes);
        bulk_load(w_smem + wsi * C::W_STAGE, wsrc, bytes, &w_full[wsi]);
        ++issued;
      }
      if (!ok)  // drain our own copies still in flight before the CTA exits
        for (int i = max(0, issued - C::W_ST); i < issued; ++i)
          mbar_wait(&w_full[i % C::W_ST], (i / C::W_ST) & 1, nullptr, 0);
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------ X producer
    if (lane == 0) {
      pdl_wait();  // activations come from the previous kernel; weights did not wait
      int issued = 0;
      bool ok = true;
      int tile = (int)(u0 / a.ksb), sb = (int)(u0 - (long)tile * a.ksb);
      for (int i = 0; i < n_units && ok; ++i, (++sb == a.ksb) ? (sb = 0, ++tile) : 0) {
        const int nt = tile % a.n_tok_tiles;
        const int xs = i % C::X_ST;
        // a tied slot is free once the unit that last used it left its A stage
        uint64_t* free_bar = C::X_TIED ? &empty[xs * C::HALVES + C::HALVES - 1] : &x_empty[xs];
        if (!(ok = mbar_wait(free_bar, ((i / C::X_ST) & 1) ^ 1, a.status, 12, i, 0))) break;
        mbar_arrive_expect_tx(&x_full[xs], C::X_UNIT_BYTES);
        uint8_t* dst = x_smem + xs * C::X_UNIT_BYTES;
#pragma unroll
        for (int c = 0; c < 4; ++c)
          tma_load_2d(dst + c * (N * 128), &x_map, sb * 256 + c * 64, nt * N, &x_full[xs]);
        QTRACE(a.trace, i, 1);
        ++issued;
      }
      if (!ok)
        for (int i = max(0, issued - C::X_ST); i < issued; ++i)
          mbar_wait(&x_full[i % C::X_ST], (i / C::X_ST) & 1, nullptr, 0);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(128, N, /*f16*/ 0);
      // Descriptor of each X stage; per-MMA K offsets are compile-time adds to
      // the start-address field (16-byte units).
      const uint64_t xdesc0 = smem_desc(smem_u32(x_smem), 16, 1024, 2);
      int seg = 0;
      bool ok = true;
      int sb = (int)(u0 % a.ksb);
      for (int i = 0; i < n_units && ok; ++i, (++sb == a.ksb) ? (sb = 0) : 0) {
        const bool first = (i == 0) || (sb == 0);
        const bool last = (i == n_units - 1) || (sb == a.ksb - 1);
        if (first && seg > 0) {
          if (!(ok = mbar_wait(d_empty, (seg - 1) & 1, a.status, 21, i, seg))) break;
        }
        const int s = i % C::U;
        const int xs = i % C::X_ST;
        if (!(ok = mbar_wait(&x_full[xs], (i / C::X_ST) & 1, a.status, 23, i, 0))) break;
        const uint64_t xd = xdesc0 + (uint64_t)((xs * C::X_UNIT_BYTES) >> 4);
        const uint32_t ab = tmem_base + C::A_COL + s * 128;
        constexpr int KPH = 16 / C::HALVES;   // MMAs per hand-off
#pragma unroll
        for (int h = 0; h < C::HALVES; ++h) {
          if (!(ok = mbar_wait(&ready[s * C::HALVES + h], (i / C::U) & 1, a.status, 22, i, h)))
            break;
          if (h == 0) QTRACE(a.trace, i, 5);
          tc_fence_after();
#pragma unroll
          for (int k8 = 0; k8 < KPH; ++k8) {
            const int kk = KPH * h + k8;
            const uint32_t acc = (uint32_t)((kk % C::NACC) * N);
            if (SWARMLLM_QGEMM_EXPERIMENT != 2)
            umma_f16_ts(tmem_base + acc, ab + kk * 8,
                        xd + (uint64_t)((((kk >> 2) * (N * 128)) + (kk & 3) * 32) >> 4), idesc,
                        (first && kk < C::NACC) ? 0u : 1u);
          }
          umma_commit(&empty[s * C::HALVES + h]);
        }
        if (!ok) break;
        if (!C::X_TIED) umma_commit(&x_empty[xs]);
        if (last) {
          umma_commit(d_full);
          ++seg;
        }
        QTRACE(a.trace, i, 6);
      }
      // All MMAs issued by this thread have completed once done_bar flips.
      umma_commit(done_bar);
      mbar_wait(done_bar, 0, nullptr, 0);
    }
  } else {
    // ------------------------------------------------------------ dequant + epilogue
    const int g = (warp - C::FIRST_DQ_WARP) >> 2;  // warpgroup
    const int quad = warp & 3;                       // TMEM lane quadrant this warp may touch
    const int row = quad * 32 + lane;                // weight row inside the 128-row tile
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    unsigned long long* tr = ((warp - C::FIRST_DQ_WARP) % 4 == 0) ? a.trace : nullptr;
    int seg = 0;
    bool ok = true;
    int tile = (int)(u0 / a.ksb), sb = (int)(u0 - (long)tile * a.ksb);
    for (int i = 0; i < n_units && ok; ++i, (++sb == a.ksb) ? (sb = 0, ++tile) : 0) {
      const bool last = (i == n_units - 1) || (sb == a.ksb - 1);
      if ((i % C::DQ) == g) {
        const int wsi = i % C::W_ST;
        if (!(ok = mbar_wait_warp(&w_full[wsi], (i / C::W_ST) & 1, a.status, 31, i, 0))) break;
        if (lane == 0) QTRACE(tr, i, 2);
        const int s = i % C::U;
        const uint32_t taddr = tmem_base + lane_off + C::A_COL + s * 128;
        const uint32_t par = ((i / C::U) & 1) ^ 1;
        const uint8_t* stage = w_smem + wsi * C::W_STAGE;
        constexpr int H = C::HALVES;
        if (kMixed && tile / a.n_tok_tiles >= a.split_tile)
          ok = dq_unit_fmt<FB, H>(stage, row, &w_empty[wsi], &empty[s * H], &ready[s * H], par,
                                  taddr, a.status, i, lane);
        else
          ok = dq_unit_fmt<F, H>(stage, row, &w_empty[wsi], &empty[s * H], &ready[s * H], par,
                                 taddr, a.status, i, lane);
        if (!ok) break;
        if (lane == 0) QTRACE(tr, i, 3);
      }
      if (last) {
        // Warpgroup 0 drains every segment.  Alternating drainers would let a
        // warpgroup wait on d_full two phases ahead after a one-unit segment,
        // where a parity wait passes too early.
        if (g == 0) {
          if (!(ok = mbar_wait_warp(d_full, seg & 1, a.status, 33, i, seg))) break;
          tc_fence_after();
          const int nt = tile % a.n_tok_tiles;
          const int n_valid = min(N, a.T - nt * N);
          const size_t off = ((size_t)(tile + blockIdx.x) * N) * 128 + row;
#pragma unroll 1
          for (int c = 0; c < N / 16; ++c) {
            uint32_t r[16];
            tmem_ld_x16(tmem_base + lane_off + c * 16, r);
            tmem_wait_ld();
#pragma unroll
            for (int acc = 1; acc < C::NACC; ++acc) {
              uint32_t r2[16];
              tmem_ld_x16(tmem_base + lane_off + acc * N + c * 16, r2);
              tmem_wait_ld();
#pragma unroll
              for (int e = 0; e < 16; ++e)
                r[e] = __float_as_uint(__uint_as_float(r[e]) + __uint_as_float(r2[e]));
            }
            if (a.n_peers == 0) {
              float* dst = a.ws + off;
#pragma unroll
              for (int e = 0; e < 16; ++e)
                if (c * 16 + e < n_valid) dst[(size_t)(c * 16 + e) * 128] = __uint_as_float(r[e]);
            } else {
              const int rt = tile / a.n_tok_tiles;
              const int o0 = a.owner_tiles > 0 ? rt / a.owner_tiles : 0;
              const int o1 = a.owner_tiles > 0 ? o0 + 1 : a.n_peers;
              for (int o = o0; o < o1; ++o) {
                float* dst = reinterpret_cast<float*>(a.peer_ws[o]) + off;
#pragma unroll
                for (int e = 0; e < 16; ++e)
                  if (c * 16 + e < n_valid)
                    dst[(size_t)(c * 16 + e) * 128] = __uint_as_float(r[e]);
              }
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(d_empty);
        }
        ++seg;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  if (a.sig_ctl != nullptr)
    ep_grid_done_signal(a.sig_ctl, a.sig_bases, a.sig_flag_off, a.n_peers, a.sig_rank);
}

// GGUF Q4_K [rows][K/256 blocks] -> tiled, nibble-permuted layout
// [rows_pad/128][K/256][128][144].  Padding rows are zero.
__global__ void q4k_repack_kernel(const uint8_t* __restrict__ src, int rows, int rows_pad, int K,
                                  uint8_t* __restrict__ dst) {
  const int ksb = K / 256;
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)rows_pad * ksb) return;
  const int r = (int)(idx / ksb), sb = (int)(idx - (long)r * ksb);
  uint8_t* out = dst + (((size_t)(r >> 7) * ksb + sb) * 128 + (r & 127)) * kQ4kRowBytes;
  if (r >= rows) {
    for (int i = 0; i < kQ4kRowBytes; ++i) out[i] = 0;
    return;
  }
  const uint8_t* b = src + ((size_t)r * ksb + sb) * 144;
  const uint8_t* qs = b + 16;
  // Word w covers K [8w, 8w+8); nibble p holds k = 8w + perm[p], perm = 0,2,4,6,1,3,5,7.
  for (int w = 0; w < 32; ++w) {
    uint32_t word = 0;
    for (int p = 0; p < 8; ++p) {
      const int kk = 8 * w + ((p < 4) ? 2 * p : 2 * (p - 4) + 1);
      const int g = kk >> 6, rr = kk & 63;
      const uint8_t byte = qs[32 * g + (rr & 31)];
      const uint32_t q = (rr < 32) ? (byte & 0xF) : (byte >> 4);
      word |= q << (4 * p);
    }
    reinterpret_cast<uint32_t*>(out)[w] = word;
  }
  for (int i = 0; i < 16; ++i) out[128 + i] = b[i];
}

// GGUF Q6_K [rows][K/256][210 B] -> [rows_pad/128][K/256][128][224 B] (qfmt.cuh).
__global__ void q6k_repack_kernel(const uint8_t* __restrict__ src, int rows, int rows_pad, int K,
                                  uint8_t* __restrict__ dst) {
  const int ksb = K / 256;
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)rows_pad * ksb) return;
  const int r = (int)(idx / ksb), sb = (int)(idx - (long)r * ksb);
  uint32_t* out = reinterpret_cast<uint32_t*>(
      dst + (((size_t)(r >> 7) * ksb + sb) * 128 + (r & 127)) * kQ6kRowBytes);
  if (r >= rows) {
    for (int i = 0; i < kQ6kRowBytes / 4; ++i) out[i] = 0;
    return;
  }
  const uint8_t* b = src + ((size_t)r * ksb + sb) * 210;
  const uint8_t* ql = b;
  const uint8_t* qh = b + 128;
  const int8_t* sc = reinterpret_cast<const int8_t*>(b + 192);
  const float d = __half2float(__ushort_as_half((uint16_t)(b[208] | (b[209] << 8))));
  // 6-bit code of value k: the low nibble comes from ql, the top two bits from qh
  // (each 128-value half: quarter q of the half uses ql bytes [64n + 32(q&1), +32),
  // nibble q>>1, and qh bits 2q..2q+1 of byte 32n + l).
  auto code = [&](int k) -> uint32_t {
    const int n = k >> 7, rr = k & 127, qt = rr >> 5, l = rr & 31;
    const uint8_t lb = ql[64 * n + 32 * (qt & 1) + l];
    const uint32_t lo = (qt >> 1) ? (lb >> 4) : (lb & 0xF);
    const uint32_t hi = (qh[32 * n + l] >> (2 * qt)) & 3;
    return lo | (hi << 4);
  };
  for (int w = 0; w < 32; ++w) {   // low nibbles, nibble order 0,2,4,6,1,3,5,7
    uint32_t word = 0;
    for (int p = 0; p < 8; ++p) {
      const int k = 8 * w + ((p < 4) ? 2 * p : 2 * (p - 4) + 1);
      word |= (code(k) & 0xF) << (4 * p);
    }
    out[w] = word;
  }
  for (int s = 0; s < 16; ++s) {   // crumbs
    uint32_t word = 0;
    for (int e = 0; e < 2; ++e)
      for (int j = 0; j < 4; ++j) {
        const int k = 16 * s + 8 * e + 2 * j;
        word |= (code(k) >> 4) << (8 * e + 2 * j);
        word |= (code(k + 1) >> 4) << (16 + 8 * e + 2 * j);
      }
    out[32 + s] = word;
  }
  for (int s = 0; s < 16; s += 2) {   // fp16 d * sc, clamped to the fp16 range
    const float a0 = fminf(fmaxf(d * (float)sc[s], -65504.f), 65504.f);
    const float a1 = fminf(fmaxf(d * (float)sc[s + 1], -65504.f), 65504.f);
    out[48 + s / 2] = (uint32_t)__half_as_ushort(__float2half_rn(a0)) |
                      ((uint32_t)__half_as_ushort(__float2half_rn(a1)) << 16);
  }
}

// GGUF Q8_0 [rows][K/32][34 B] -> [rows_pad/128][K/256][128][272 B] (qfmt.cuh):
// codes as q ^ 0x80, then the superblock's 8 fp16 block scales.
__global__ void q80_repack_kernel(const uint8_t* __restrict__ src, int rows, int rows_pad, int K,
                                  uint8_t* __restrict__ dst) {
  const int ksb = K / 256;
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)rows_pad * ksb) return;
  const int r = (int)(idx / ksb), sb = (int)(idx - (long)r * ksb);
  uint8_t* out = dst + (((size_t)(r >> 7) * ksb + sb) * 128 + (r & 127)) * kQ80RowBytes;
  if (r >= rows) {
    for (int i = 0; i < kQ80RowBytes; ++i) out[i] = 0;
    return;
  }
  const uint8_t* b = src + ((size_t)r * (K / 32) + sb * 8) * 34;
  for (int blk = 0; blk < 8; ++blk) {
    const uint8_t* q = b + blk * 34;
    for (int i = 0; i < 32; ++i) out[blk * 32 + i] = q[2 + i] ^ 0x80;
    out[256 + 2 * blk] = q[0];
    out[256 + 2 * blk + 1] = q[1];
  }
}

}  // namespace swarm

using namespace swarm;

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)p;
  }
  return fn;
}

// 2D fp16/bf16 row-major tensor [rows, cols] (row stride in elements), box
// {box_cols, box_rows}, 128 B swizzle when box_cols * 2 == 128.
int make_tmap_2d_16bit(CUtensorMap* map, const void* base, int rows, int cols, int row_stride,
                       int box_rows, int box_cols, int swizzle_bytes) {
  EncodeTiledFn enc = get_encode_tiled();
  if (!enc) return -1;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_stride * 2};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  CUtensorMapSwizzle sw = swizzle_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                          : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                          : swizzle_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                                : CU_TENSOR_MAP_SWIZZLE_NONE;
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims,
                   strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

static unsigned long long* g_trace = nullptr;

// Debug: record the event timeline of CTA 0 of every following launch into
// `buf` (device, >= 512*8 u64); nullptr turns it off.
void qgemm_set_trace(void* buf) { g_trace = static_cast<unsigned long long*>(buf); }

int q4k_tc_tok_tile(int T) {
  if (T <= 16) return 16;
  if (T <= 32) return 32;
  if (T <= 64) return 64;
  return 128;  // N=128 already runs the tensor core at full rate (48..69 clk per K=16 MMA)
}

static int q_env(const char* name, int dflt) {
  const char* v = getenv(name);
  return v ? atoi(v) : dflt;
}

static const bool g_pdl = q_env("SWARMLLM_PDL", 1) != 0;
bool swarm::pdl_enabled() { return g_pdl; }
static const int g_gemv_max_t = [] {
  const int v = q_env("SWARMLLM_QGEMV_MAX_T", kQGemvMaxT);
  return v < 0 ? 0 : (v > kQGemvMaxT ? kQGemvMaxT : v);
}();
int q4k_gemv_max_t() { return g_gemv_max_t; }

int q4k_plan_max_ctas(int T, int num_sms, int fmt) {
  return T <= g_gemv_max_t ? qgemv_ctas_per_sm(fmt, T) * num_sms : num_sms;
}

// Work decomposition shared by the launcher, the workspace sizing and GemmOut.
// At <= q4k_gemv_max_t() tokens the units go to the GEMV's CTAs instead (same
// partial-slot format, token tile 16).
void q4k_tc_plan(int rows, int K, int T, int num_sms, int* tok_tile, int* n_tok_tiles, int* ksb,
                 long* total_units, int* upc, int* n_ctas, size_t* ws_floats, int fmt) {
  const int N = q4k_tc_tok_tile(T);
  const int ntt = (T + N - 1) / N;
  const int kb = K / 256;
  const int tiles = ((rows + 127) / 128) * ntt;
  const long total = (long)tiles * kb;
  const int max_ctas = q4k_plan_max_ctas(T, num_sms, fmt);
  const int u = (int)((total + max_ctas - 1) / max_ctas);
  const int ctas = (int)((total + u - 1) / u);
  *tok_tile = N;
  *n_tok_tiles = ntt;
  *ksb = kb;
  *total_units = total;
  *upc = u;
  *n_ctas = ctas;
  *ws_floats = (size_t)(tiles + ctas) * N * 128;
}

template <class F, class FB, int N>
static int launch_n(const CUtensorMap& map, const QGemmArgs& a, int n_ctas, cudaStream_t s) {
  using C = QCfg<F, FB, N>;
  static unsigned long long attr_done = 0;
  if (!smem_attr_once(qgemm_q4k_tc_kernel<F, FB, N>, C::SMEM, &attr_done)) return -3;
  if (launch_pdl(qgemm_q4k_tc_kernel<F, FB, N>, dim3(n_ctas), dim3(C::THREADS), C::SMEM, s, map,
                 a) != cudaSuccess)
    return -4;
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}

template <class F, class FB = F>
static int launch_f(int N, const CUtensorMap& map, const QGemmArgs& a, int n_ctas,
                    cudaStream_t s) {
  switch (N) {
    case 16: return launch_n<F, FB, 16>(map, a, n_ctas, s);
    case 32: return launch_n<F, FB, 32>(map, a, n_ctas, s);
    case 64: return launch_n<F, FB, 64>(map, a, n_ctas, s);
    default: return launch_n<F, FB, 128>(map, a, n_ctas, s);
  }
}


int launch_qgemm_q4k_tc(const void* w_packed, int rows, int K, const __half* x, int x_stride,
                        int T, float* ws, size_t ws_floats_avail, int num_sms, int* status,
                        GemmOut* out, cudaStream_t s, const unsigned long long* peer_ws,
                        int n_peers, int* sig_ctl, const unsigned long long* sig_bases,
                        long long sig_flag_off, int sig_rank, int owner_tiles, int fmt,
                        const void* w_b, int fmt_b, int split_tile) {
  if (T <= 0) return 0;
  if (K % 256 != 0 || rows % 128 != 0 || fmt < 0 || fmt >= kNumQFmts) return -1;
  const bool mixed = w_b != nullptr && fmt_b >= 0 && fmt_b != fmt;
  if (mixed && !(fmt == kFmtQ4K && fmt_b == kFmtQ6K)) return -1;   // the Q4_K_M q|k|v mix
  if (mixed && (split_tile <= 0 || split_tile >= rows / 128)) return -1;
  // the GEMV's resident CTAs per SM follow the wider format's stages
  const int plan_fmt = mixed && qfmt_row_bytes(fmt_b) > qfmt_row_bytes(fmt) ? fmt_b : fmt;
  if ((x_stride % 8) != 0 || (reinterpret_cast<uintptr_t>(x) & 15) != 0) return -5;
  int N, ntt, kb, upc, ctas;
  long total;
  size_t need;
  q4k_tc_plan(rows, K, T, num_sms, &N, &ntt, &kb, &total, &upc, &ctas, &need, plan_fmt);
  if (need > ws_floats_avail) return -6;
  if (total >= (1L << 24)) return -8;   // GemmOut's segment lookup assumes fewer units
  if (out) {
    out->ws = ws;
    out->rows = rows;
    out->T = T;
    out->mode = 1;
    out->ksb = kb;
    out->upc = upc;
    out->tok_tile = N;
    out->n_tok_tiles = ntt;
    out->seg_max = 0;
    gemm_out_finalize(out);
  }
  if (T <= g_gemv_max_t)
    return launch_qgemv_q4k(w_packed, rows, K, x, x_stride, T, ws, kb, total, upc, ctas, status,
                            peer_ws, n_peers, sig_ctl, sig_bases, sig_flag_off, sig_rank, s,
                            owner_tiles, fmt, mixed ? w_b : nullptr, mixed ? fmt_b : -1,
                            split_tile);
  CUtensorMap map;
  if (make_tmap_2d_16bit(&map, x, T, K, x_stride, N, 64, 128) != 0) return -2;
  QGemmArgs a{(const uint8_t*)w_packed, (const uint8_t*)w_b, mixed ? split_tile : 0, rows, K, T,
              ntt, kb, total, upc, ws, status, g_trace};
  a.n_peers = 0;
  a.owner_tiles = 0;
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
  if (mixed) return launch_f<FmtQ4K, FmtQ6K>(N, map, a, ctas, s);
  switch (fmt) {
    case kFmtQ4K: return launch_f<FmtQ4K>(N, map, a, ctas, s);
    case kFmtQ6K: return launch_f<FmtQ6K>(N, map, a, ctas, s);
    default: return launch_f<FmtQ80>(N, map, a, ctas, s);
  }
}

int launch_q4k_repack(const void* src, int rows, int K, void* dst, cudaStream_t s) {
  const int rows_pad = (rows + 127) / 128 * 128;
  const long n = (long)rows_pad * (K / 256);
  q4k_repack_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>((const uint8_t*)src, rows,
                                                                 rows_pad, K, (uint8_t*)dst);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

int launch_qfmt_repack(int fmt, const void* src, int rows, int K, void* dst, cudaStream_t s) {
  if (fmt == kFmtQ4K) return launch_q4k_repack(src, rows, K, dst, s);
  if ((fmt != kFmtQ6K && fmt != kFmtQ8_0) || K % 256 != 0) return -1;
  const int rows_pad = (rows + 127) / 128 * 128;
  const long n = (long)rows_pad * (K / 256);
  const unsigned grid = (unsigned)((n + 127) / 128);
  if (fmt == kFmtQ6K)
    q6k_repack_kernel<<<grid, 128, 0, s>>>((const uint8_t*)src, rows, rows_pad, K, (uint8_t*)dst);
  else
    q80_repack_kernel<<<grid, 128, 0, s>>>((const uint8_t*)src, rows, rows_pad, K, (uint8_t*)dst);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}
