// Paged attention on tcgen05 tensor cores: decode, draft-tree verification and
// chunked prefill in one kernel.
//
// One CTA = one "row group" x one KV head x one key split.  A row group is up
// to 128 MMA rows made of (query position, GQA head) pairs of one sequence:
// e.g. 16 prefill positions x 8 query heads per KV head, or 1 decode position
// x 8 heads.  Per 128-key tile (8 fp16 pages of 16 tokens, fetched by TMA):
//
//   S  = Q K^T          tcgen05.mma  A=Q (smem, K-major)  B=K tile (smem, K-major)
//   softmax             one thread per row: masks (causal length, sliding
//                       window, draft-tree ancestor bits), online max/sum
//   P  -> TMEM (fp16)   tcgen05.st
//   O += P V            tcgen05.mma  A=P (TMEM)  B=V tile (smem, MN-major)
//
// For head_dim <= 128, S and P are double-buffered in TMEM and the MMA thread
// issues QK^T of tile j+1 before P V of tile j, so the tensor core works while
// the softmax of the previous tile runs.
//
// The fp32 O accumulator stays in TMEM; a row is rescaled in TMEM only when its
// running max moves.  With one split the kernel finishes the softmax (adding
// learned sinks) and writes fp16 output; with several it writes (O, max, sum)
// partials that decode_attn_combine merges.
//
// Replaces the reference's decode_attn_f16kv / tree_attn_tiled_f16kv and its
// FA2 sm80 prefill (kernels/decode_attn.cu:109,311;
// vendor/candle-flash-attn/kernels/flash_fwd_kernel.h), which read a
// contiguous per-request cache with mma.sync/SIMT math.
// Cache layout: [pages][n_kv][16][head_dim] fp16.
#include "kernels.h"
#include "tc_utils.cuh"

namespace swarm {
using namespace tc;

constexpr int kAttnKeys = 128;  // keys per tile
constexpr int kPageTok = 16;

template <int D>
struct AttnCfg {
  static constexpr int DH = D / 64;                       // 128-byte column blocks of d
  static constexpr int Q_BYTES = 128 * D * 2;             // 128 rows
  static constexpr int KV_TILE = kAttnKeys * D * 2;       // K or V tile
  static constexpr int ST = D <= 64 ? 4 : (D <= 128 ? 3 : 1);  // K/V tile stages
  static constexpr int SMEM = 1024 + Q_BYTES + ST * 2 * KV_TILE + 256;
  // DB: S and P double-buffered in TMEM, so QK^T of tile j+1 runs while the
  // softmax of tile j does (needs D <= 128 for the columns).
  static constexpr bool DB = D <= 128;
  static constexpr int NB = DB ? 2 : 1;
  __host__ __device__ static constexpr int s_col(int b) { return b * 128; }
  __host__ __device__ static constexpr int p_col(int b) { return DB ? 256 + b * 64 : 128; }
  static constexpr int O_COL = DB ? 384 : 256;
  static constexpr int THREADS = 192;                     // 4 softmax warps, producer, MMA
  static_assert(O_COL + D <= 512, "TMEM");
  static_assert(SMEM <= 227 * 1024, "smem");
};

struct AttnTcArgs {
  const int32_t* group_row0;   // [G] first token row of each group
  const int32_t* group_npos;   // [G] positions in the group
  const int32_t* block_table;  // [T, bt_stride]
  int bt_stride;
  const int32_t* seq_lens;     // [T] visible keys per row
  const uint64_t* tree_mask;   // [T] or null
  const int32_t* tree_start;   // [T] or null
  const float* sinks;          // [n_q] or null
  int n_q, n_kv, n_rep, pos_per_group;
  int window;
  float scale_log2;            // softmax scale * log2(e)
  int keys_per_split, n_splits;
  __half* out;                 // [T, n_q, D]   (n_splits == 1)
  float* part_o;               // [T, n_q, n_splits, D]
  float* part_ml;              // [T, n_q, n_splits, 2]
  int* status;
  unsigned long long* trace;   // debug: per-tile event timestamps of CTA (0,0,0)
};

// Debug timeline of CTA (0,0,0) (see attn_set_trace); compiled in only with
// -DSWARMLLM_KERNEL_TRACE (setup.py: SWARMLLM_KERNEL_TRACE=1).
#ifdef SWARMLLM_KERNEL_TRACE
#define ATRACE(a, j, ev)                                                                      \
  do {                                                                                       \
    if ((a).trace && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && (j) < 64)      \
      (a).trace[(j) * 8 + (ev)] = globaltimer();                                             \
  } while (0)
#else
#define ATRACE(a, j, ev) \
  do {                   \
  } while (0)
#endif

SW_DEVICE float exp2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int D, bool TREE, int REP>
__global__ void __launch_bounds__(192, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap q_map, const __grid_constant__ CUtensorMap k_map,
                   const __grid_constant__ CUtensorMap v_map, AttnTcArgs a) {
  pdl_trigger();  // dependents (the next GEMM) may launch and prefetch weights
  pdl_wait();     // what earlier kernels wrote is complete and visible
  using C = AttnCfg<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* q_s = smem;
  uint8_t* kv_s = smem + C::Q_BYTES;  // stage st: K at st*2*KV_TILE, V after it
  uint64_t* bars = reinterpret_cast<uint64_t*>(kv_s + C::ST * 2 * C::KV_TILE);
  uint64_t* q_full = bars;
  uint64_t* kv_full = q_full + 1;          // [ST]
  uint64_t* kv_empty = kv_full + C::ST;    // [ST]
  uint64_t* s_full = kv_empty + C::ST;     // [NB] QK done
  uint64_t* p_full = s_full + C::NB;       // [NB] P written (4 warps)
  uint64_t* pv_done = p_full + C::NB;      // PV done (one phase per tile)
  uint64_t* o_done = pv_done + 1;          // every MMA of the CTA done (one phase)
  uint64_t* rep_done = o_done + 1;         // replica partials staged (4 softmax warps)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rep_done + 1);

  const int g = blockIdx.x, hk = blockIdx.y, sp = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = a.group_row0[g], npos = a.group_npos[g];
  const int nrows = npos * a.n_rep;
  const int l_max = a.seq_lens[row0 + npos - 1];
  int k_lo = sp * a.keys_per_split;
  const int k_hi = min(l_max, k_lo + a.keys_per_split);
  if (a.window > 0) {
    const int l_min = a.seq_lens[row0];
    k_lo = max(k_lo, max(0, l_min - a.window) / kAttnKeys * kAttnKeys);
  }
  const int n_tiles = k_hi > k_lo ? (k_hi - k_lo + kAttnKeys - 1) / kAttnKeys : 0;
  const int32_t* bt = a.block_table + (size_t)row0 * a.bt_stride;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < C::ST; ++i) { mbar_init(&kv_full[i], 1); mbar_init(&kv_empty[i], 1); }
    for (int b = 0; b < C::NB; ++b) { mbar_init(&s_full[b], 1); mbar_init(&p_full[b], 4); }
    mbar_init(pv_done, 1);
    mbar_init(o_done, 1);
    mbar_init(rep_done, 4);
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0 && n_tiles > 0) {
      prefetch_tensormap(&q_map);
      prefetch_tensormap(&k_map);
      prefetch_tensormap(&v_map);
      // REP copies of the group's 8 rows, one per TMEM lane quadrant (rows
      // 32k.., 4096-byte offsets, so the 128-byte swizzle of every copy matches)
      mbar_arrive_expect_tx(q_full, (uint32_t)(REP * C::DH * a.n_rep * a.pos_per_group * 128));
#pragma unroll
      for (int dh = 0; dh < C::DH; ++dh)
#pragma unroll
        for (int k = 0; k < REP; ++k)
          tma_load_3d(q_s + dh * 128 * 128 + k * 4096, &q_map, dh * 64, hk * a.n_rep, row0, q_full);
      // Page ids of the next tile are read before waiting for a free stage, all
      // eight at once (the TMA asm is a compiler memory barrier, so reading them
      // inside the issue loop would serialise eight L2 round trips per tile).
      constexpr int kPages = kAttnKeys / kPageTok;
      int pg[kPages];
      auto fetch_pages = [&](int j) {
        const int b0 = (k_lo + j * kAttnKeys) / kPageTok;
#pragma unroll
        for (int p = 0; p < kPages; ++p) pg[p] = (b0 + p < a.bt_stride) ? __ldg(bt + b0 + p) : 0;
      };
      fetch_pages(0);
      for (int j = 0; j < n_tiles; ++j) {
        const int st = j % C::ST;
        int cur[kPages];
#pragma unroll
        for (int p = 0; p < kPages; ++p) cur[p] = pg[p];
        if (j + 1 < n_tiles) fetch_pages(j + 1);
        if (!mbar_wait(&kv_empty[st], ((j / C::ST) & 1) ^ 1, a.status, 41, j, 0)) break;
        uint8_t* ks = kv_s + st * 2 * C::KV_TILE;
        uint8_t* vs = ks + C::KV_TILE;
        // Always 8 whole pages: keys past the end are masked, and a full load keeps
        // stale-but-finite data out of the P.V product.
        ATRACE(a, j, 0);
        mbar_arrive_expect_tx(&kv_full[st], (uint32_t)(2 * C::KV_TILE));
#pragma unroll
        for (int p = 0; p < kPages; ++p) {
          const int r = (cur[p] * a.n_kv + hk) * kPageTok;
#pragma unroll
          for (int dh = 0; dh < C::DH; ++dh) {
            tma_load_2d(ks + dh * kAttnKeys * 128 + p * kPageTok * 128, &k_map, dh * 64, r, &kv_full[st]);
            tma_load_2d(vs + dh * kAttnKeys * 128 + p * kPageTok * 128, &v_map, dh * 64, r, &kv_full[st]);
          }
        }
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && n_tiles > 0) {
      const uint32_t idesc_qk = idesc_f16(128, kAttnKeys, 0);
      const uint32_t idesc_pv = idesc_f16(128, D, 0, /*a_mn*/ 0, /*b_mn*/ 1);
      const uint64_t qd = smem_desc(smem_u32(q_s), 16, 1024, 2);
      bool ok = mbar_wait(q_full, 0, a.status, 42, 0, 0);
      // S(j) = Q K(j)^T into S buffer b  (K over the head dim)
      auto issue_qk = [&](int j) -> bool {
        const int st = j % C::ST;
        if (!mbar_wait(&kv_full[st], (j / C::ST) & 1, a.status, 43, j, 0)) return false;
        ATRACE(a, j, 1);
        tc_fence_after();
        const uint64_t kd = smem_desc(smem_u32(kv_s + st * 2 * C::KV_TILE), 16, 1024, 2);
        const int b = C::DB ? (j & 1) : 0;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t off = (uint64_t)((((kk >> 2) * (kAttnKeys * 128)) + (kk & 3) * 32) >> 4);
          const uint64_t qoff = (uint64_t)((((kk >> 2) * (128 * 128)) + (kk & 3) * 32) >> 4);
          umma_f16_ss(tmem + C::s_col(b), qd + qoff, kd + off, idesc_qk, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[b]);
        ATRACE(a, j, 2);
        return true;
      };
      // With DB, QK(j+1) is issued before PV(j): its S buffer was last read by
      // the softmax of tile j-1, which finished before PV(j-1) was issued.
      if (C::DB && ok && n_tiles > 0) ok = issue_qk(0);
      for (int j = 0; j < n_tiles && ok; ++j) {
        const int st = j % C::ST;
        if (C::DB) {
          if (j + 1 < n_tiles && !(ok = issue_qk(j + 1))) break;
        } else {
          if (!(ok = issue_qk(j))) break;
        }
        // O += P V  (K over keys); V tile is MN-major: LBO = d-block stride, SBO = 8 keys
        const int b = C::DB ? (j & 1) : 0;
        if (!(ok = mbar_wait(&p_full[b], C::DB ? ((j >> 1) & 1) : (j & 1), a.status, 44, j, 0))) break;
        ATRACE(a, j, 5);
        tc_fence_after();
        const uint32_t kb = smem_u32(kv_s + st * 2 * C::KV_TILE);
        const uint64_t vd = smem_desc(kb + C::KV_TILE, kAttnKeys * 128, 1024, 2);
#pragma unroll
        for (int kk = 0; kk < kAttnKeys / 16; ++kk)
          umma_f16_ts(tmem + C::O_COL, tmem + C::p_col(b) + kk * 8,
                      vd + (uint64_t)((kk * 16 * 128) >> 4), idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(pv_done);
        umma_commit(&kv_empty[st]);
      }
      umma_commit(o_done);   // tracks everything this thread issued
    }
  } else {
    // ------------------------------------------------------------ softmax (thread = row)
    // REP == 4 (groups of exactly 8 rows, i.e. one decode position x 8 query
    // heads): Q was loaded once per TMEM lane quadrant, so lanes 0..7 of every
    // softmax warp hold the group's rows, and warp q owns keys [32q, 32q+32) of
    // every tile (its P rows are zero elsewhere).  tcgen05.ld/st take one
    // column address per warp, which is why a replica is a warp, not a lane.
    // Each replica keeps its own running max and sum, so tiles need no
    // cross-warp traffic; the four are merged like key-split partials at the
    // end.  The softmax work of a tile is then spread over four schedulers
    // and is a quarter as long.
    constexpr int KW = kAttnKeys / REP;  // keys of a tile owned by one warp
    const int m = threadIdx.x;           // TMEM lane / MMA row 0..127
    const int rrow = REP == 1 ? m : lane;
    const int kq = REP == 1 ? 0 : warp;
    const int quad = warp;      // warps 0..3 -> TMEM lane quadrants 0..3
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const bool real = REP == 1 ? (m < nrows) : (lane < 8);
    const bool warp_real = __any_sync(0xffffffffu, real);
    const int pi = real ? rrow / a.n_rep : 0;
    const int h = real ? rrow - pi * a.n_rep : 0;
    const int trow = row0 + pi;
    const int L = real ? a.seq_lens[trow] : 0;
    const int lo_win = (a.window > 0) ? max(0, L - a.window) : 0;
    const uint64_t tmask = (real && TREE) ? a.tree_mask[trow] : ~0ull;
    const int tstart = (real && TREE) ? a.tree_start[trow] : 0x7fffffff;
    // m_run: the max P is computed against.  It is raised lazily (only when a
    // new score exceeds it by more than 2^8 in the log2 domain), so P <= 256
    // stays in fp16 range and O is rescaled in TMEM only a few times per row.
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    if (REP > 1) {  // P rows start zero: each replica writes only its keys
      uint32_t z[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) z[e] = 0u;
#pragma unroll
      for (int b = 0; b < C::NB; ++b)
#pragma unroll
        for (int c = 0; c < kAttnKeys / 32; ++c) tmem_st_x16(tmem + lane_off + C::p_col(b) + c * 16, z);
      tmem_wait_st();
    }
    for (int j = 0; j < n_tiles && ok; ++j) {
      // Without DB, s_full(j) also covers PV(j-1): a commit tracks all of the MMA
      // thread's earlier tcgen05 operations.  With DB it covers PV(j-2), which
      // is what reusing P buffer (j & 1) needs.
      const int b = C::DB ? (j & 1) : 0;
      if (!(ok = mbar_wait_warp(&s_full[b], C::DB ? ((j >> 1) & 1) : (j & 1), a.status, 45, j, 0)))
        break;
      if (threadIdx.x == 0) ATRACE(a, j, 3);
      if (warp_real) {
        tc_fence_after();
        const int key0 = k_lo + j * kAttnKeys + kq * KW;
        float s[KW];
#pragma unroll
        for (int c = 0; c < KW / 16; ++c)
          tmem_ld_x16(tmem + lane_off + C::s_col(b) + kq * KW + c * 16,
                      reinterpret_cast<uint32_t*>(s) + c * 16);
        tmem_wait_ld();
        // visible keys of this row inside its window: [vlo, vhi) (+ tree bits)
        const int vlo = max(lo_win - key0, 0), vhi = min(L - key0, KW);
        float mt = -INFINITY;
        const bool full = !TREE && __all_sync(0xffffffffu, vlo == 0 && vhi == KW);
        if (full) {  // whole window visible for every row of the warp: no masking
#pragma unroll
          for (int c = 0; c < KW; ++c) {
            s[c] *= a.scale_log2;
            mt = fmaxf(mt, s[c]);
          }
        } else {
#pragma unroll
          for (int c = 0; c < KW; ++c) {
            bool vis = c >= vlo && c < vhi;
            if (TREE) {
              const int k = key0 + c;
              if (k >= tstart) vis = vis && (k - tstart) < 64 && ((tmask >> (k - tstart)) & 1ull);
            }
            s[c] = vis ? s[c] * a.scale_log2 : -INFINITY;
            mt = fmaxf(mt, s[c]);
          }
        }
        float m_new = m_run;
        if (m_run == -INFINITY) {
          m_new = mt;  // nothing accumulated yet: O and l are zero
        } else if (mt > m_run + 8.f) {
          m_new = mt;
        }
        if (__any_sync(0xffffffffu, m_new != m_run && m_run != -INFINITY)) {
          // With DB, PV(j-1) may still be accumulating into O: wait for it.  (s_full(j)
          // implies PV(j-2) is done, so pv_done is at most one phase behind here.)
          if (C::DB && j > 0) {
            if (!(ok = mbar_wait_warp(pv_done, (j - 1) & 1, a.status, 46, j, 0))) break;
            tc_fence_after();
          }
          const float alpha = (m_new != m_run && m_run != -INFINITY) ? exp2_approx(m_run - m_new) : 1.f;
          l_run *= alpha;
#pragma unroll 1
          for (int c = 0; c < D / 16; ++c) {
            uint32_t o[16];
            tmem_ld_x16(tmem + lane_off + C::O_COL + c * 16, o);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tmem_st_x16(tmem + lane_off + C::O_COL + c * 16, o);
          }
        }
        m_run = m_new;
        float ls = 0.f;
        uint32_t pk[KW / 2];
        // exp2(-inf - m) = 0, so masked keys need no special case (m_run is
        // finite whenever any key of the row is visible; otherwise all s are
        // -inf and m_run = -inf: clamp to keep p = 0 instead of NaN).
        const float msub = (m_run == -INFINITY) ? 0.f : m_run;
#pragma unroll
        for (int c = 0; c < KW; c += 2) {
          const float p0 = exp2_approx(s[c] - msub);
          const float p1 = exp2_approx(s[c + 1] - msub);
          ls += p0 + p1;
          __half2 hp = __floats2half2_rn(p0, p1);
          pk[c / 2] = *reinterpret_cast<uint32_t*>(&hp);
        }
        l_run += ls;
#pragma unroll
        for (int c = 0; c < KW / 32; ++c)
          tmem_st_x16(tmem + lane_off + C::p_col(b) + kq * (KW / 2) + c * 16, pk + c * 16);
        tmem_wait_st();
        tc_fence_before();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[b]);
      if (threadIdx.x == 0) ATRACE(a, j, 4);
    }
    // ---- finish: wait for the last PV, then write output or partials
    if (ok && n_tiles > 0)
      ok = C::DB ? mbar_wait_warp(o_done, 0, a.status, 47, 0, 0)
                 : mbar_wait_warp(pv_done, (n_tiles - 1) & 1, a.status, 47, 0, 0);
    if (ok) tc_fence_after();
    if (REP > 1) {
      // ---- merge the four replicas (warps) of each row through shared memory
      // (the K/V stages are idle now: every tile was consumed before o_done)
      float* red = reinterpret_cast<float*>(kv_s);          // [REP][8][2]  (max, sum)
      float* obuf = red + REP * 8 * 2;                        // [REP][8][D]
      if (real) {
        red[(kq * 8 + lane) * 2 + 0] = m_run;
        red[(kq * 8 + lane) * 2 + 1] = l_run;
      }
#pragma unroll 1
      for (int c = 0; c < D / 16; ++c) {
        uint32_t o[16];
        if (n_tiles > 0) {
          tmem_ld_x16(tmem + lane_off + C::O_COL + c * 16, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) o[e] = 0u;
        }
        if (real) {
#pragma unroll
          for (int e = 0; e < 16; ++e) obuf[(kq * 8 + lane) * D + c * 16 + e] = __uint_as_float(o[e]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(rep_done);
      const bool merged_ok = mbar_wait(rep_done, 0, a.status, 48, 0, 0);
      // thread t: row t / 16, dims [(t % 16) * D / 16, +D / 16)
      const int r = m >> 4, dd = (m & 15) * (D / 16);
      float M = -INFINITY;
#pragma unroll
      for (int k = 0; k < REP; ++k) M = fmaxf(M, red[(k * 8 + r) * 2]);
      float f[REP], l = 0.f;
#pragma unroll
      for (int k = 0; k < REP; ++k) {
        const float mk = red[(k * 8 + r) * 2];
        f[k] = (mk == -INFINITY) ? 0.f : exp2_approx(mk - M);
        l += f[k] * red[(k * 8 + r) * 2 + 1];
      }
      const int hq = hk * a.n_rep + r;
      if (merged_ok && a.n_splits == 1) {
        float oscale = 1.f;
        if (a.sinks) {
          const float sk = a.sinks[hq] * 1.4426950408889634f;
          const float mm = fmaxf(M, sk);
          const float fm = (M == -INFINITY) ? 0.f : exp2_approx(M - mm);
          l = l * fm + exp2_approx(sk - mm);
          oscale = fm;
        }
        const float inv = l > 0.f ? oscale / l : 0.f;
        __half* dst = a.out + ((size_t)row0 * a.n_q + hq) * D + dd;
#pragma unroll
        for (int e = 0; e < D / 16; e += 2) {
          float v0 = 0.f, v1 = 0.f;
#pragma unroll
          for (int k = 0; k < REP; ++k) {
            v0 += f[k] * obuf[(k * 8 + r) * D + dd + e];
            v1 += f[k] * obuf[(k * 8 + r) * D + dd + e + 1];
          }
          *reinterpret_cast<__half2*>(dst + e) = __floats2half2_rn(v0 * inv, v1 * inv);
        }
      } else if (merged_ok) {
        const size_t pb = ((size_t)row0 * a.n_q + hq) * a.n_splits + sp;
        float* po = a.part_o + pb * D + dd;
#pragma unroll
        for (int e = 0; e < D / 16; ++e) {
          float v = 0.f;
#pragma unroll
          for (int k = 0; k < REP; ++k) v += f[k] * obuf[(k * 8 + r) * D + dd + e];
          po[e] = v;
        }
        if ((m & 15) == 0) {
          a.part_ml[pb * 2 + 0] = (n_tiles > 0 && M != -INFINITY) ? M * 0.6931471805599453f : -INFINITY;
          a.part_ml[pb * 2 + 1] = l;
        }
      }
    } else {
    const int hq = hk * a.n_rep + h;
    if (warp_real && a.n_splits == 1) {
      float oscale = 1.f;
      if (a.sinks && real) {
        const float sk = a.sinks[hq] * 1.4426950408889634f;  // sink logit in the log2 domain
        const float mm = fmaxf(m_run, sk);
        const float f = (m_run == -INFINITY) ? 0.f : exp2_approx(m_run - mm);
        l_run = l_run * f + exp2_approx(sk - mm);
        oscale = f;
      }
      const float inv = l_run > 0.f ? oscale / l_run : 0.f;
      __half* dst = a.out + ((size_t)trow * a.n_q + hq) * D;
#pragma unroll 1
      for (int c = 0; c < D / 16; ++c) {
        uint32_t o[16];
        if (n_tiles > 0) {
          tmem_ld_x16(tmem + lane_off + C::O_COL + c * 16, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) o[e] = 0u;
        }
        if (real) {
#pragma unroll
          for (int e = 0; e < 16; e += 2)
            *reinterpret_cast<__half2*>(dst + c * 16 + e) =
                __floats2half2_rn(__uint_as_float(o[e]) * inv, __uint_as_float(o[e + 1]) * inv);
        }
      }
    } else if (warp_real) {
      const size_t pb = ((size_t)trow * a.n_q + hq) * a.n_splits + sp;
      float* po = a.part_o + pb * D;
#pragma unroll 1
      for (int c = 0; c < D / 16 && n_tiles > 0; ++c) {
        uint32_t o[16];
        tmem_ld_x16(tmem + lane_off + C::O_COL + c * 16, o);
        tmem_wait_ld();
        if (real) {
#pragma unroll
          for (int e = 0; e < 16; ++e) po[c * 16 + e] = __uint_as_float(o[e]);
        }
      }
      if (real) {
        // partials in natural-log units, as the combine kernel expects
        a.part_ml[pb * 2 + 0] = (n_tiles > 0 && m_run != -INFINITY) ? m_run * 0.6931471805599453f : -INFINITY;
        a.part_ml[pb * 2 + 1] = l_run;
      }
    }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace swarm

using namespace swarm;

typedef CUresult (*EncodeTiledFn2)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn2 encode_fn() {
  static EncodeTiledFn2 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn2)p;
  }
  return fn;
}

// q: [T, n_q, D] -> 3D map {D, n_q, T}, box {64, n_rep, pos_per_group}
static int make_q_map(CUtensorMap* m, const __half* q, int T, int n_q, int D, int n_rep, int ppg) {
  auto enc = encode_fn();
  if (!enc) return -1;
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)n_q, (cuuint64_t)T};
  cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)n_q * D * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)n_rep, (cuuint32_t)ppg};
  cuuint32_t es[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half*>(q), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
             ? 0 : -2;
}

// cache: [pages, n_kv, 16, D] viewed as 2D rows x D, box {64, 16}
static int make_kv_map(CUtensorMap* m, const __half* cache, long rows, int D) {
  auto enc = encode_fn();
  if (!enc) return -1;
  cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)D * 2};
  cuuint32_t box[2] = {64, 16};
  cuuint32_t es[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(cache), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
             ? 0 : -2;
}

static unsigned long long* g_attn_trace = nullptr;
void attn_set_trace(void* buf) { g_attn_trace = static_cast<unsigned long long*>(buf); }

template <int D>
static int launch_d(const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm,
                    const AttnTcArgs& a, int G, cudaStream_t s) {
  using C = AttnCfg<D>;
  static unsigned long long done1 = 0, done_tree = 0, done4 = 0;
  if (!smem_attr_once(attn_tc_kernel<D, false, 1>, C::SMEM, &done1) ||
      !smem_attr_once(attn_tc_kernel<D, true, 1>, C::SMEM, &done_tree) ||
      !smem_attr_once(attn_tc_kernel<D, false, 4>, C::SMEM, &done4))
    return -3;
  dim3 grid(G, a.n_kv, a.n_splits);
  cudaError_t e;
  if (a.tree_mask != nullptr)
    e = launch_pdl(attn_tc_kernel<D, true, 1>, grid, dim3(C::THREADS), C::SMEM, s, qm, km, vm, a);
  else if (a.n_rep * a.pos_per_group == 8)  // 8-row groups (decode, 8 heads per KV head)
    e = launch_pdl(attn_tc_kernel<D, false, 4>, grid, dim3(C::THREADS), C::SMEM, s, qm, km, vm, a);
  else
    e = launch_pdl(attn_tc_kernel<D, false, 1>, grid, dim3(C::THREADS), C::SMEM, s, qm, km, vm, a);
  if (e != cudaSuccess) return -4;
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}

int launch_attn_tc(const __half* q, int T, int n_q, const __half* k_cache, const __half* v_cache,
                   long num_pages, int n_kv, int D, const int32_t* group_row0,
                   const int32_t* group_npos, int G, int pos_per_group, const int32_t* block_table,
                   int bt_stride, const int32_t* seq_lens, const uint64_t* tree_mask,
                   const int32_t* tree_start, const float* sinks, int window, float scale,
                   int keys_per_split, int n_splits, __half* out, float* part_o, float* part_ml,
                   int* status, cudaStream_t s) {
  if (G <= 0) return 0;
  const int n_rep = n_q / n_kv;
  if (n_rep * pos_per_group > 128 || keys_per_split % kAttnKeys) return -5;
  CUtensorMap qm, km, vm;
  if (make_q_map(&qm, q, T, n_q, D, n_rep, pos_per_group)) return -2;
  const long rows = num_pages * n_kv * kPageTok;
  if (make_kv_map(&km, k_cache, rows, D) || make_kv_map(&vm, v_cache, rows, D)) return -2;
  AttnTcArgs a{group_row0, group_npos, block_table, bt_stride, seq_lens, tree_mask, tree_start,
               sinks, n_q, n_kv, n_rep, pos_per_group, window, scale * 1.4426950408889634f,
               keys_per_split, n_splits, out, part_o, part_ml, status, g_attn_trace};
  switch (D) {
    case 64: return launch_d<64>(qm, km, vm, a, G, s);
    case 128: return launch_d<128>(qm, km, vm, a, G, s);
    case 256: return launch_d<256>(qm, km, vm, a, G, s);
    default: return -6;
  }
}
