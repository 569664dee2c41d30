// Chunked gated delta rule for prefill (same recurrence as delta_rule in
// deltanet.cu, evaluated 64 tokens at a time).
//
// Within a chunk with entering state S0 [dk][dv], cumulative log-decay
// G_t = g_1 + ... + g_t and gamma_t = exp(G_t), unrolling the recurrence gives
//   S_t   = gamma_t S0 + sum_{s<=t} exp(G_t - G_s) k_s d_s^T
//   d_t   = beta_t (v_t - gamma_t S0^T k_t - sum_{s<t} exp(G_t - G_s)(k_t.k_s) d_s)
// i.e. (I + A) D = diag(beta) V - diag(beta gamma) K S0 with the strictly lower
// triangular A[t][s] = beta_t exp(G_t - G_s) (k_t.k_s).  Solving
//   (I + A) U = diag(beta) V,   (I + A) W = diag(beta gamma) K
// gives D = U - W S0, then
//   O     = diag(gamma) Q S0 + (Mask o exp(G_t - G_s) o Q K^T) D
//   S_new = gamma_L S0 + (K o exp(G_L - G_t))^T D.
// All decay factors are <= 1 (g <= 0), so nothing overflows.  The value
// columns of S evolve independently, so one CTA owns (sequence, value head,
// 32-column group): 4x the CTAs of the recurrent kernel; the chunks of one
// sequence run in order inside the CTA.  The triangular solves run one right-
// hand-side column per thread with the column held in registers (no barrier
// per row).  The head output (before the gated RMSNorm, which needs the whole
// head) goes to an fp32 buffer; gated_norm finishes it.
//
// Reference: the recurrence of kernels/delta_rule.cu:212 (the reference has
// only the token-sequential form; chunked evaluation is listed as not done in
// its docs/ARCHITECTURE.md:964).
#include "kernels.h"
#include "gemm_out.cuh"
#include "common.cuh"

namespace swarm {

constexpr int kCh = 64;          // tokens per chunk
constexpr int kDk = 128;         // key head dim
constexpr int kDvg = 32;         // value columns per CTA
constexpr int kPk = kDk + 1;     // padded row pitch of Q/K/W (bank-conflict free)
constexpr int kChunkThreads = 256;

struct ChunkSmem {
  float q[kCh][kPk];
  float k[kCh][kPk];
  float w[kCh][kPk];
  float v[kCh][kDvg];
  float u[kCh][kDvg];   // U, then D
  float a[kCh][kCh];    // A (strictly lower)
  float m[kCh][kCh];    // masked decayed Q K^T
  float s0[kDk][kDvg];
  float G[kCh], beta[kCh], red[2][8];
};

__global__ void __launch_bounds__(kChunkThreads, 1) delta_chunk_kernel(
    const float* __restrict__ qkv, int C, int nk, int nv, GemmOut gba,
    const float* __restrict__ dt_bias, const float* __restrict__ Aa, float* __restrict__ state,
    const int4* __restrict__ seqs, float* __restrict__ o_raw) {
  extern __shared__ __align__(16) uint8_t chunk_smem_raw[];
  ChunkSmem& sm = *reinterpret_cast<ChunkSmem*>(chunk_smem_raw);
  const int s = blockIdx.x, h = blockIdx.y, cg = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int4 sq = seqs[s];
  const int r0 = sq.x, n = sq.y, slot = sq.z, p0 = sq.w;
  if (n <= 0) return;
  const int kh = h / (nv / nk);
  const float qscale = rsqrtf((float)kDk);
  float* st = state + ((size_t)slot * nv + h) * kDk * kDk;  // [dk][dv]
  for (int e = tid; e < kDk * kDvg; e += kChunkThreads) {
    const int i = e / kDvg, j = e % kDvg;
    sm.s0[i][j] = p0 == 0 ? 0.f : st[(size_t)i * kDk + cg * kDvg + j];
  }
  const float Ah = Aa[h], dtb = dt_bias[h];
  for (int c0 = 0; c0 < n; c0 += kCh) {
    const int L = min(kCh, n - c0);
    // ---- load rows: L2-normalised q (scaled) and k, this CTA's v columns, gates
    for (int t = warp; t < kCh; t += kChunkThreads / 32) {
      float qv[4], kv[4];
      float qq = 0.f, kk = 0.f;
      const bool valid = t < L;
      const float* xr = qkv + (size_t)(r0 + c0 + t) * C;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = lane + 32 * e;
        qv[e] = valid ? xr[kh * kDk + i] : 0.f;
        kv[e] = valid ? xr[nk * kDk + kh * kDk + i] : 0.f;
        qq += qv[e] * qv[e];
        kk += kv[e] * kv[e];
      }
      qq = warp_sum(qq);
      kk = warp_sum(kk);
      const float iq = rsqrtf(qq + 1e-6f) * qscale, ik = rsqrtf(kk + 1e-6f);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        sm.q[t][lane + 32 * e] = qv[e] * iq;
        sm.k[t][lane + 32 * e] = kv[e] * ik;
      }
      sm.v[t][lane] = valid ? xr[2 * nk * kDk + h * kDk + cg * kDvg + lane] : 0.f;
    }
    // gates: one row per thread, so the 64 rows' partial-sum reads are in flight together
    if (tid < kCh) {
      const int t = tid;
      float b = 0.f, gdec = 0.f;
      if (t < L) {
        const int row = r0 + c0 + t;
        const float bl = gba.get(row, h), al = gba.get(row, nv + h) + dtb;
        b = 1.f / (1.f + __expf(-bl));
        gdec = Ah * (al > 20.f ? al : log1pf(__expf(al)));
      }
      sm.beta[t] = b;
      sm.G[t] = gdec;
    }
    __syncthreads();
    if (warp == 0) {  // inclusive prefix sum of the log decays (64 values, 2 per lane)
      float g0 = sm.G[2 * lane], g1 = sm.G[2 * lane + 1];
      float pair = g0 + g1, incl = pair;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      const float excl = incl - pair;
      sm.G[2 * lane] = excl + g0;
      sm.G[2 * lane + 1] = excl + g0 + g1;
    }
    __syncthreads();
    // ---- A (strictly lower) and the masked decayed Q K^T (lower incl. diagonal):
    //      a 4 x 4 register tile per thread, rows tb + 16a, columns ub + 16b (with the
    //      129-float row pitch both operand loads are bank-conflict free)
    {
      const int tb = tid >> 4, ub = tid & 15;
      float dk[4][4], dq[4][4];
#pragma unroll
      for (int x = 0; x < 4; ++x)
#pragma unroll
        for (int y = 0; y < 4; ++y) dk[x][y] = dq[x][y] = 0.f;
#pragma unroll 4
      for (int i = 0; i < kDk; ++i) {
        float kt[4], qt[4], ku[4];
#pragma unroll
        for (int x = 0; x < 4; ++x) {
          kt[x] = sm.k[tb + 16 * x][i];
          qt[x] = sm.q[tb + 16 * x][i];
          ku[x] = sm.k[ub + 16 * x][i];
        }
#pragma unroll
        for (int x = 0; x < 4; ++x)
#pragma unroll
          for (int y = 0; y < 4; ++y) {
            dk[x][y] += kt[x] * ku[y];
            dq[x][y] += qt[x] * ku[y];
          }
      }
#pragma unroll
      for (int x = 0; x < 4; ++x)
#pragma unroll
        for (int y = 0; y < 4; ++y) {
          const int t = tb + 16 * x, u = ub + 16 * y;
          float av = 0.f, mv = 0.f;
          if (u <= t) {
            const float dec = __expf(sm.G[t] - sm.G[u]);
            mv = dec * dq[x][y];
            if (u < t) av = sm.beta[t] * dec * dk[x][y];
          }
          sm.a[t][u] = av;
          sm.m[t][u] = mv;
        }
    }
    __syncthreads();
    // ---- forward substitution, one right-hand-side column per thread:
    //      threads 0..127 -> W columns (rhs beta gamma k), 128..159 -> U columns (rhs beta v)
    if (tid < kDk + kDvg) {
      float x[kCh];
      const bool isw = tid < kDk;
      const int col = isw ? tid : tid - kDk;
#pragma unroll
      for (int t = 0; t < kCh; ++t) {
        float b = isw ? sm.beta[t] * __expf(sm.G[t]) * sm.k[t][col] : sm.beta[t] * sm.v[t][col];
#pragma unroll
        for (int u = 0; u < t; ++u) b -= sm.a[t][u] * x[u];
        x[t] = b;
      }
#pragma unroll
      for (int t = 0; t < kCh; ++t) {
        if (isw) sm.w[t][col] = x[t];
        else sm.u[t][col] = x[t];
      }
    }
    __syncthreads();
    // ---- D = U - W S0 (in place in u): a 2 x 4 tile per thread, rows tb, tb + 32,
    //      columns jb + 8c
    {
      const int tb = tid >> 3, jb = tid & 7;
      float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll 4
      for (int i = 0; i < kDk; ++i) {
        const float w0 = sm.w[tb][i], w1 = sm.w[tb + 32][i];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float sv = sm.s0[i][jb + 8 * c];
          acc[0][c] += w0 * sv;
          acc[1][c] += w1 * sv;
        }
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        sm.u[tb][jb + 8 * c] -= acc[0][c];
        sm.u[tb + 32][jb + 8 * c] -= acc[1][c];
      }
    }
    __syncthreads();
    // ---- O = gamma Q S0 + M D -> o_raw (same tiling; M is zero above the diagonal,
    //      so the u loop runs to the warp's last row)
    {
      const int tb = tid >> 3, jb = tid & 7;
      const int uend = min(kCh, ((tid >> 5) << 2) + 36);
      float qs[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      float md[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll 4
      for (int i = 0; i < kDk; ++i) {
        const float q0 = sm.q[tb][i], q1 = sm.q[tb + 32][i];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float sv = sm.s0[i][jb + 8 * c];
          qs[0][c] += q0 * sv;
          qs[1][c] += q1 * sv;
        }
      }
#pragma unroll 4
      for (int u = 0; u < uend; ++u) {
        const float m0 = sm.m[tb][u], m1 = sm.m[tb + 32][u];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float dv = sm.u[u][jb + 8 * c];
          md[0][c] += m0 * dv;
          md[1][c] += m1 * dv;
        }
      }
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int t = tb + 32 * r;
        if (t < L) {
          const float gt = __expf(sm.G[t]);
#pragma unroll
          for (int c = 0; c < 4; ++c)
            o_raw[(size_t)(r0 + c0 + t) * nv * kDk + h * kDk + cg * kDvg + jb + 8 * c] =
                gt * qs[r][c] + md[r][c];
        }
      }
    }
    __syncthreads();
    // ---- S0 <- gamma_L S0 + sum_t exp(G_L - G_t) k_t d_t^T: scale the rows of D by
    //      exp(G_L - G_t), then a 4 x 4 tile per thread, rows ib + 32a, columns jb + 8c
    {
      const float GL = sm.G[L - 1];
      for (int e = tid; e < kCh * kDvg; e += kChunkThreads) {
        const int t = e / kDvg, j = e % kDvg;
        sm.u[t][j] *= __expf(GL - sm.G[t]);
      }
      __syncthreads();
      const int ib = tid >> 3, jb = tid & 7;
      const float gl = __expf(GL);
      float acc[4][4];
#pragma unroll
      for (int x = 0; x < 4; ++x)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[x][c] = gl * sm.s0[ib + 32 * x][jb + 8 * c];
#pragma unroll 4
      for (int t = 0; t < L; ++t) {
        float kv[4], dv[4];
#pragma unroll
        for (int x = 0; x < 4; ++x) kv[x] = sm.k[t][ib + 32 * x];
#pragma unroll
        for (int c = 0; c < 4; ++c) dv[c] = sm.u[t][jb + 8 * c];
#pragma unroll
        for (int x = 0; x < 4; ++x)
#pragma unroll
          for (int c = 0; c < 4; ++c) acc[x][c] += kv[x] * dv[c];
      }
#pragma unroll
      for (int x = 0; x < 4; ++x)
#pragma unroll
        for (int c = 0; c < 4; ++c) sm.s0[ib + 32 * x][jb + 8 * c] = acc[x][c];
    }
    __syncthreads();
  }
  for (int e = tid; e < kDk * kDvg; e += kChunkThreads) {
    const int i = e / kDvg, j = e % kDvg;
    st[(size_t)i * kDk + cg * kDvg + j] = sm.s0[i][j];
  }
}

// One warp per (row, head): rmsnorm(o) * w * silu(z) -> fp16.
__global__ void gated_norm_kernel(const float* __restrict__ o_raw, GemmOut gz,
                                  const float* __restrict__ norm_w, float eps, int T, int nv,
                                  __half* __restrict__ out) {
  pdl_trigger();  // dependents (the next GEMM) may launch and prefetch weights
  pdl_wait();     // what earlier kernels wrote is complete and visible
  const int idx = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (idx >= T * nv) return;
  const int row = idx / nv, h = idx % nv;
  const float* o = o_raw + (size_t)row * nv * kDk + h * kDk;
  float v[4], ss = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    v[e] = o[lane + 32 * e];
    ss += v[e] * v[e];
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / kDk + eps);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int j = lane + 32 * e;
    out[(size_t)row * nv * kDk + h * kDk + j] =
        __float2half_rn(v[e] * inv * norm_w[j] * silu(gz.get(row, h * kDk + j)));
  }
}

}  // namespace swarm

using namespace swarm;

int launch_delta_chunk(const float* qkv, int C, int nk, int nv, int D, const GemmOut& gba,
                       const float* dt_bias, const float* A, const GemmOut& gz,
                       const float* norm_w, float eps, float* state, const void* seqs, int S,
                       int T, float* o_raw, __half* out, cudaStream_t s) {
  if (S <= 0 || T <= 0) return 0;
  if (D != kDk || nv % nk) return -1;
  const int smem = (int)sizeof(ChunkSmem);
  static unsigned long long attr_done = 0;
  if (!smem_attr_once(delta_chunk_kernel, smem, &attr_done)) return -3;
  delta_chunk_kernel<<<dim3(S, nv, kDk / kDvg), kChunkThreads, smem, s>>>(
      qkv, C, nk, nv, gba, dt_bias, A, state, (const int4*)seqs, o_raw);
  const int warps = T * nv;
  gated_norm_kernel<<<(warps + 7) / 8, 256, 0, s>>>(o_raw, gz, norm_w, eps, T, nv, out);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -2;
}
