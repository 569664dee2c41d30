// Dense fp16 x fp16 GEMM on the 5th-generation tensor cores for 16-bit weight
// matrices (BF16/F16 checkpoints: gpt-oss attention and LM head, routers of
// shared experts, ...):
//
//   out[t][r] = sum_k W[r][k] * X[t][k],   W: fp16 [rows, K], X: fp16 [T, K]
//
// Same contract as the Q4_K kernel (qgemm_tc.cu): swap-AB (M = 128 weight rows,
// N = token tile 16..128), persistent stream-K over (row tile, token tile,
// 128-wide K unit) with one fp32 partial per touched tile in the workspace, so
// every GEMM epilogue kernel (gemm_out.cuh) reads it unchanged.  Both operands
// arrive by TMA (128 B swizzle, K-major) and the MMA reads them from shared
// memory; the accumulator is double-buffered in TMEM so the epilogue warps
// drain one tile segment while the next accumulates.  K need not be a multiple
// of the unit: TMA fills the out-of-range columns of both operands with zeros.
//
// Warps: 0 = TMA producer, 1 = TMEM owner + MMA issuer, 2..5 = epilogue.
// Replaces the reference's dequantize-to-f16 + cuBLAS path for 16-bit weights
// (vendor/candle/candle-core/src/quantized/cuda.rs:1005).
#include "kernels.h"
#include "gemm_out.cuh"
#include "tc_utils.cuh"

namespace swarm {
using namespace tc;

template <int N>
struct DCfg {
  static constexpr int ST = N == 128 ? 3 : 4;
  static constexpr int W_STAGE = 128 * 128 * 2;  // 128 rows x 128 K
  static constexpr int X_STAGE = N * 128 * 2;
  static constexpr int THREADS = 192;
  static constexpr int SMEM = 1024 + ST * (W_STAGE + X_STAGE) + 256;
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
};

struct DGemmArgs {
  int rows, K, T, n_tok_tiles, kb;
  long total_units;
  int upc;
  float* ws;
  int* status;
};

template <int N>
__global__ void __launch_bounds__(DCfg<N>::THREADS, 1)
    dense_gemm_tc_kernel(const __grid_constant__ CUtensorMap w_map,
                         const __grid_constant__ CUtensorMap x_map, DGemmArgs a) {
  using C = DCfg<N>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* w_smem = smem;
  uint8_t* x_smem = smem + C::ST * C::W_STAGE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(x_smem + C::ST * C::X_STAGE);
  uint64_t* full = bars;
  uint64_t* empty = full + C::ST;
  uint64_t* d_full = empty + C::ST;  // [2]
  uint64_t* d_empty = d_full + 2;    // [2]
  uint64_t* done_bar = d_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long u0 = (long)blockIdx.x * a.upc;
  const long u1 = min(a.total_units, u0 + a.upc);
  const int n_units = (int)max(0L, u1 - u0);

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::ST; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(&d_full[i], 1); mbar_init(&d_empty[i], 4); }
    mbar_init(done_bar, 1);
    fence_barrier_init();
    prefetch_tensormap(&w_map);
    prefetch_tensormap(&x_map);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      bool ok = true;
      int tile = (int)(u0 / a.kb), kb = (int)(u0 - (long)tile * a.kb);
      for (int i = 0; i < n_units && ok; ++i, (++kb == a.kb) ? (kb = 0, ++tile) : 0) {
        const int rt = tile / a.n_tok_tiles, nt = tile - rt * a.n_tok_tiles;
        const int s = i % C::ST;
        if (!(ok = mbar_wait(&empty[s], ((i / C::ST) & 1) ^ 1, a.status, 51, i, 0))) break;
        mbar_arrive_expect_tx(&full[s], C::W_STAGE + C::X_STAGE);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          tma_load_2d(w_smem + s * C::W_STAGE + c * (128 * 128), &w_map, kb * 128 + c * 64,
                      rt * 128, &full[s]);
          tma_load_2d(x_smem + s * C::X_STAGE + c * (N * 128), &x_map, kb * 128 + c * 64,
                      nt * N, &full[s]);
        }
        ++issued;
      }
      if (!ok)
        for (int i = max(0, issued - C::ST); i < issued; ++i)
          mbar_wait(&full[i % C::ST], (i / C::ST) & 1, nullptr, 0);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(128, N, 0);
      const uint64_t wdesc0 = smem_desc(smem_u32(w_smem), 16, 1024, 2);
      const uint64_t xdesc0 = smem_desc(smem_u32(x_smem), 16, 1024, 2);
      int seg = 0;
      bool ok = true;
      int kb = (int)(u0 % a.kb);
      for (int i = 0; i < n_units && ok; ++i, (++kb == a.kb) ? (kb = 0) : 0) {
        const bool first = (i == 0) || (kb == 0);
        const bool last = (i == n_units - 1) || (kb == a.kb - 1);
        const int slot = seg & 1;
        if (first && seg >= 2) {
          if (!(ok = mbar_wait(&d_empty[slot], ((seg >> 1) - 1) & 1, a.status, 52, i, seg))) break;
        }
        const int s = i % C::ST;
        if (!(ok = mbar_wait(&full[s], (i / C::ST) & 1, a.status, 53, i, 0))) break;
        tc_fence_after();
        const uint64_t wd = wdesc0 + (uint64_t)((s * C::W_STAGE) >> 4);
        const uint64_t xd = xdesc0 + (uint64_t)((s * C::X_STAGE) >> 4);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_f16_ss(tmem_base + slot * N,
                      wd + (uint64_t)((((kk >> 2) * (128 * 128)) + (kk & 3) * 32) >> 4),
                      xd + (uint64_t)((((kk >> 2) * (N * 128)) + (kk & 3) * 32) >> 4), idesc,
                      (first && kk == 0) ? 0u : 1u);
        umma_commit(&empty[s]);
        if (last) {
          umma_commit(&d_full[slot]);
          ++seg;
        }
      }
      umma_commit(done_bar);
      mbar_wait(done_bar, 0, nullptr, 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    int seg = 0;
    bool ok = true;
    int tile = (int)(u0 / a.kb), kb = (int)(u0 - (long)tile * a.kb);
    for (int i = 0; i < n_units && ok; ++i, (++kb == a.kb) ? (kb = 0, ++tile) : 0) {
      const bool last = (i == n_units - 1) || (kb == a.kb - 1);
      if (!last) continue;
      const int slot = seg & 1;
      if (!(ok = mbar_wait_warp(&d_full[slot], (seg >> 1) & 1, a.status, 54, i, seg))) break;
      tc_fence_after();
      const int nt = tile % a.n_tok_tiles;
      const int n_valid = min(N, a.T - nt * N);
      float* dst = a.ws + ((size_t)(tile + blockIdx.x) * N) * 128 + row;
#pragma unroll 1
      for (int c = 0; c < N / 16; ++c) {
        uint32_t r[16];
        tmem_ld_x16(tmem_base + lane_off + slot * N + c * 16, r);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 16; ++e)
          if (c * 16 + e < n_valid) dst[(size_t)(c * 16 + e) * 128] = __uint_as_float(r[e]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&d_empty[slot]);
      ++seg;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, 256);
  }
}

}  // namespace swarm

using namespace swarm;

void dense_tc_plan(int rows, int K, int T, int num_sms, int* tok_tile, int* n_tok_tiles, int* kb,
                   long* total_units, int* upc, int* n_ctas, size_t* ws_floats) {
  const int N = q4k_tc_tok_tile(T);
  const int ntt = (T + N - 1) / N;
  const int kbn = (K + 127) / 128;
  const int tiles = ((rows + 127) / 128) * ntt;
  const long total = (long)tiles * kbn;
  const int u = (int)((total + num_sms - 1) / num_sms);
  const int ctas = (int)((total + u - 1) / u);
  *tok_tile = N;
  *n_tok_tiles = ntt;
  *kb = kbn;
  *total_units = total;
  *upc = u;
  *n_ctas = ctas;
  *ws_floats = (size_t)(tiles + ctas) * N * 128;
}

template <int N>
static int dense_launch_n(const CUtensorMap& wm, const CUtensorMap& xm, const DGemmArgs& a,
                          int ctas, cudaStream_t s) {
  using C = DCfg<N>;
  static unsigned long long attr_done = 0;
  if (!smem_attr_once(dense_gemm_tc_kernel<N>, C::SMEM, &attr_done)) return -3;
  dense_gemm_tc_kernel<N><<<ctas, C::THREADS, C::SMEM, s>>>(wm, xm, a);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}

int launch_dense_gemm_tc(const __half* w, int rows, int K, int w_stride, const __half* x,
                         int x_stride, int T, float* ws, size_t ws_floats_avail, int num_sms,
                         int* status, GemmOut* out, cudaStream_t s) {
  if (T <= 0) return 0;
  if (K % 8 || w_stride % 8 || x_stride % 8) return -1;
  if ((reinterpret_cast<uintptr_t>(w) & 15) || (reinterpret_cast<uintptr_t>(x) & 15)) return -5;
  int N, ntt, kb, upc, ctas;
  long total;
  size_t need;
  dense_tc_plan(rows, K, T, num_sms, &N, &ntt, &kb, &total, &upc, &ctas, &need);
  if (need > ws_floats_avail) return -6;
  if (total >= (1L << 24)) return -8;   // GemmOut's segment lookup assumes fewer units
  CUtensorMap wm, xm;
  if (make_tmap_2d_16bit(&wm, w, rows, K, w_stride, 128, 64, 128) != 0) return -2;
  if (make_tmap_2d_16bit(&xm, x, T, K, x_stride, N, 64, 128) != 0) return -2;
  DGemmArgs a{rows, K, T, ntt, kb, total, upc, ws, status};
  int rc;
  switch (N) {
    case 16: rc = dense_launch_n<16>(wm, xm, a, ctas, s); break;
    case 32: rc = dense_launch_n<32>(wm, xm, a, ctas, s); break;
    case 64: rc = dense_launch_n<64>(wm, xm, a, ctas, s); break;
    default: rc = dense_launch_n<128>(wm, xm, a, ctas, s); break;
  }
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
  return rc;
}
