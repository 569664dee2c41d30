// Paged attention and the SwiGLU tail on the host CPU.
//
// cpu_paged_attention: every (block of up to 16 tokens of one sequence, KV
// head) pair is one OpenMP task that serves all the query heads sharing that
// KV head, so a key/value row is converted to fp32 once per block and group,
// not once per query head and token.  Keys are
// walked in 256-key chunks: the chunk's scores for all the group's heads are
// computed first (scale, optional tanh soft-cap, sliding window and the
// 64-bit draft-tree visibility mask applied), then one online-softmax update
// (running max, rescaled sum and accumulator) folds the chunk in.  Attention
// sinks join the denominator at the end as one more logit per head.  The
// reference computes the same rows in its CPU split path
// (src/inference/split/attn_rows.rs, attn_softmax.rs, prefill_attn.rs).
//
// exp is evaluated as 2^n e^r: n = round(x / ln 2) goes into the float's
// exponent field, r = x - n ln 2 is reduced in two steps (Cody-Waite) and e^r
// on |r| <= ln2 / 2 is its degree-6 Taylor series (relative error below 5e-7),
// written so the compiler vectorises it (the reference keeps its own AVX2 expf
// in src/inference/fast_math.rs).
#include "cpu_attn.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

// The hot loops are compiled for three x86-64 levels (AVX-512, AVX2, baseline)
// and the loader picks the best the CPU has.
#define SWARM_CLONES __attribute__((target_clones("arch=x86-64-v4", "arch=x86-64-v3", "default")))

namespace swarm_native {
namespace {

constexpr int kChunk = 256;

// fp16 -> fp32 without branches, so a row converts in vector registers: the
// 15 magnitude bits moved to the float's exponent/mantissa position are the
// value times 2^-112 (subnormal halves land on float subnormals, exactly),
// so one multiply by 2^112 rescales; exponent 31 (inf / NaN) is patched.
__attribute__((always_inline)) inline float half_to_float(uint16_t h) {
  const uint32_t mag = (uint32_t)(h & 0x7FFF) << 13;
  float f;
  std::memcpy(&f, &mag, 4);
  f *= 5.192296858534828e33f;  // 2^112
  uint32_t bits;
  std::memcpy(&bits, &f, 4);
  bits = (h & 0x7C00) == 0x7C00 ? 0x7F800000u | mag : bits;  // inf / NaN keep their payload
  bits |= (uint32_t)(h & 0x8000) << 16;
  std::memcpy(&f, &bits, 4);
  return f;
}

}  // namespace

// Selects instead of branches and rounding by adding and subtracting
// 1.5 * 2^23 (exact to nearest for |y| < 2^22), so loops over it vectorise.
__attribute__((always_inline)) static inline float exp_fast(float x) {
  // n = round(x / ln2), r = x - n ln2 with ln2 split into a high part with a
  // short mantissa (n * hi is exact) and the remainder (Cody and Waite), so r
  // keeps full precision however large n is; e^x = 2^n e^r, |r| <= ln2 / 2.
  const bool under = x < -87.3f;
  x = x < -87.3f ? -87.3f : (x > 88.7f ? 88.7f : x);
  const float n = (x * 1.44269504088896341f + 12582912.f) - 12582912.f;
  const float r = (x - n * 0.693145751953125f) - n * 1.42860682030941723e-6f;
  float p = 1.f / 720.f;
  p = p * r + 1.f / 120.f;
  p = p * r + 1.f / 24.f;
  p = p * r + 1.f / 6.f;
  p = p * r + 0.5f;
  p = p * r + 1.f;
  p = p * r + 1.f;
  const int32_t e = ((int32_t)n + 127) << 23;
  float s;
  std::memcpy(&s, &e, 4);
  return under ? 0.f : p * s;
}

float exp_approx(float x) { return exp_fast(x); }

SWARM_CLONES static void silu_mul_span(const float* g, const float* u, float* out, int64_t i0,
                                       int64_t i1, float limit, float alpha) {
#pragma omp simd
  for (int64_t i = i0; i < i1; ++i) {
    float a = g[i], b = u[i];
    if (limit > 0.f) {  // gpt-oss: clamped gate, clamped and shifted up, sigmoid(alpha g)
      a = a < limit ? a : limit;
      b = b < -limit ? -limit : b > limit ? limit : b;
      out[i] = a / (1.f + exp_fast(-alpha * a)) * (b + 1.f);
    } else {
      out[i] = a / (1.f + exp_fast(-a)) * b;
    }
  }
}

void cpu_silu_mul(const float* g, const float* u, float* out, int64_t n, float limit, float alpha) {
  constexpr int64_t kSpan = 16384;
  const int64_t spans = (n + kSpan - 1) / kSpan;
#pragma omp parallel for schedule(static) if (spans > 4)
  for (int64_t c = 0; c < spans; ++c)
    silu_mul_span(g, u, out, c * kSpan, std::min(n, (c + 1) * kSpan), limit, alpha);
}

template <typename KV>
static inline float kv_load(const KV* p, int i);
template <>
__attribute__((always_inline)) inline float kv_load<float>(const float* p, int i) {
  return p[i];
}
template <>
__attribute__((always_inline)) inline float kv_load<uint16_t>(const uint16_t* p, int i) {
  return half_to_float(p[i]);
}

constexpr int kTokBlock = 16;   // query tokens of one sequence sharing a task

struct AttnScratch {
  float *s, *acc, *krow, *vrow, *m, *l;
};

// Tokens t0..t0+nt of one sequence (same block table) and one KV head g: all
// their query heads share each converted K / V row, so a prefill reads the
// cache once per block of up to kTokBlock tokens instead of once per token.
// Each (token, head) row keeps its own key range (window, causal length),
// tree visibility and online-softmax state.  Inlined into per-ISA clones
// (below); the OpenMP loop that hands out the tasks stays outside them, since
// OpenMP outlines its regions before functions are cloned.
template <typename KV, int NTMAX>
__attribute__((always_inline)) static inline void attn_task(const AttnArgs& a, const KV* kc,
                                                            const KV* vc, int t0, int nt_, int g,
                                                            AttnScratch& w) {
  const int nt = NTMAX == 1 ? 1 : nt_;   // a lone token (decode) compiles its own loops
  const int nq = a.n_heads, nkv = a.n_kv_heads, d = a.head_dim;
  const int rep = nq / nkv, ps = a.page_size, R = nt * rep;
  float *s = w.s, *acc = w.acc, *krow = w.krow, *vrow = w.vrow, *m = w.m, *l = w.l;
  int lo_t[NTMAX], len_t[NTMAX], ts_t[NTMAX];
  uint64_t tm_t[NTMAX];
  int lo = 1 << 30, hi = 0;
  for (int u = 0; u < nt; ++u) {
    const int t = t0 + u, Lt = a.seq_lens[t];
    len_t[u] = Lt;
    lo_t[u] = a.window > 0 && Lt > a.window ? Lt - a.window : 0;
    ts_t[u] = a.tree_start ? a.tree_start[t] : 0;
    tm_t[u] = a.tree_mask ? (uint64_t)a.tree_mask[t] : 0;
    lo = lo_t[u] < lo ? lo_t[u] : lo;
    hi = Lt > hi ? Lt : hi;
  }
  const int32_t* bt = a.block_table + (size_t)t0 * a.max_pages;
  for (int i = 0; i < R * d; ++i) acc[i] = 0.f;
  for (int r = 0; r < R; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.f;
  }
  for (int c0 = lo; c0 < hi; c0 += kChunk) {
    const int nc = hi - c0 < kChunk ? hi - c0 : kChunk;
    for (int j = 0; j < nc; ++j) {
      const int key = c0 + j;
      bool any = false;
      bool vis[NTMAX];
      for (int u = 0; u < nt; ++u) {
        bool v = key >= lo_t[u] && key < len_t[u];
        if (v && a.tree_mask) {
          const int rel = key - ts_t[u];
          v = rel < 0 || (rel < 64 && ((tm_t[u] >> rel) & 1));
        }
        vis[u] = v;
        any |= v;
      }
      if (any) {
        const size_t off =
            (((size_t)bt[key / ps] * nkv + g) * ps + (size_t)(key % ps)) * (size_t)d;
#pragma omp simd
        for (int i = 0; i < d; ++i) krow[i] = kv_load(kc + off, i);
      }
      for (int u = 0; u < nt; ++u) {
        const float* qt = a.q + ((size_t)(t0 + u) * nq + (size_t)g * rep) * d;
        for (int h = 0; h < rep; ++h) {
          float dot = -INFINITY;
          if (vis[u]) {
            const float* qh = qt + (size_t)h * d;
            dot = 0.f;
#pragma omp simd reduction(+ : dot)
            for (int i = 0; i < d; ++i) dot += qh[i] * krow[i];
            dot *= a.scale;
            if (a.softcap > 0.f) dot = a.softcap * std::tanh(dot / a.softcap);
          }
          s[(size_t)(u * rep + h) * kChunk + j] = dot;
        }
      }
    }
    for (int r = 0; r < R; ++r) {
      float* sh = s + (size_t)r * kChunk;
      float mx = m[r];
      for (int j = 0; j < nc; ++j) mx = sh[j] > mx ? sh[j] : mx;
      if (mx == -INFINITY) continue;  // nothing visible yet
      const float corr = m[r] == -INFINITY ? 0.f : exp_fast(m[r] - mx);
      float sum = 0.f;
#pragma omp simd reduction(+ : sum)
      for (int j = 0; j < nc; ++j) {
        const float p = sh[j] == -INFINITY ? 0.f : exp_fast(sh[j] - mx);
        sh[j] = p;
        sum += p;
      }
      l[r] = l[r] * corr + sum;
      m[r] = mx;
      float* ah = acc + (size_t)r * d;
      for (int i = 0; i < d; ++i) ah[i] *= corr;
    }
    for (int j = 0; j < nc; ++j) {
      bool any = false;
      for (int r = 0; r < R; ++r) any |= s[(size_t)r * kChunk + j] > 0.f;
      if (!any) continue;
      const int key = c0 + j;
      const size_t off =
          (((size_t)bt[key / ps] * nkv + g) * ps + (size_t)(key % ps)) * (size_t)d;
#pragma omp simd
      for (int i = 0; i < d; ++i) vrow[i] = kv_load(vc + off, i);
      for (int r = 0; r < R; ++r) {
        const float p = s[(size_t)r * kChunk + j];
        if (p == 0.f) continue;
        float* ah = acc + (size_t)r * d;
#pragma omp simd
        for (int i = 0; i < d; ++i) ah[i] += p * vrow[i];
      }
    }
  }
  for (int u = 0; u < nt; ++u)
    for (int h = 0; h < rep; ++h) {
      const int r = u * rep + h;
      float den = l[r], sc = 1.f;
      if (a.sinks) {
        const float sk = a.sinks[g * rep + h];
        const float mx = m[r] > sk ? m[r] : sk;
        sc = m[r] == -INFINITY ? 0.f : exp_fast(m[r] - mx);
        den = l[r] * sc + exp_fast(sk - mx);
      }
      const float inv = den > 0.f ? sc / den : 0.f;
      float* o = a.out + ((size_t)(t0 + u) * nq + (size_t)g * rep + h) * d;
      const float* ah = acc + (size_t)r * d;
      for (int i = 0; i < d; ++i) o[i] = ah[i] * inv;
    }
}

SWARM_CLONES static void attn_task_f16(const AttnArgs& a, const uint16_t* k, const uint16_t* v,
                                       int t0, int nt, int g, AttnScratch& w) {
  if (nt == 1)
    attn_task<uint16_t, 1>(a, k, v, t0, 1, g, w);
  else
    attn_task<uint16_t, kTokBlock>(a, k, v, t0, nt, g, w);
}

SWARM_CLONES static void attn_task_f32(const AttnArgs& a, const float* k, const float* v, int t0,
                                       int nt, int g, AttnScratch& w) {
  if (nt == 1)
    attn_task<float, 1>(a, k, v, t0, 1, g, w);
  else
    attn_task<float, kTokBlock>(a, k, v, t0, nt, g, w);
}

int cpu_paged_attention(const AttnArgs& a, const void* k_cache, const void* v_cache,
                        bool kv_fp16) {
  if (a.n_heads % a.n_kv_heads != 0 || a.head_dim <= 0 || a.page_size <= 0) return -1;
  const int rep = a.n_heads / a.n_kv_heads, d = a.head_dim;
  // blocks of consecutive tokens that read the same pages (one sequence)
  std::vector<int> starts;
  for (int t = 0; t < a.n_tokens; ++t) {
    const bool same = !starts.empty() && t - starts.back() < kTokBlock &&
                      std::memcmp(a.block_table + (size_t)t * a.max_pages,
                                  a.block_table + (size_t)starts.back() * a.max_pages,
                                  sizeof(int32_t) * (size_t)a.max_pages) == 0;
    if (!same) starts.push_back(t);
  }
  starts.push_back(a.n_tokens);
  const int nb = (int)starts.size() - 1, R = kTokBlock * rep;
#pragma omp parallel
  {
    std::vector<float> buf((size_t)R * kChunk + (size_t)R * d + 2 * (size_t)d + 2 * (size_t)R);
    AttnScratch w;
    w.s = buf.data();
    w.acc = w.s + (size_t)R * kChunk;
    w.krow = w.acc + (size_t)R * d;
    w.vrow = w.krow + d;
    w.m = w.vrow + d;
    w.l = w.m + R;
#pragma omp for collapse(2) schedule(dynamic)
    for (int b = 0; b < nb; ++b)
      for (int g = 0; g < a.n_kv_heads; ++g) {
        const int t0 = starts[b], nt = starts[b + 1] - starts[b];
        if (kv_fp16)
          attn_task_f16(a, static_cast<const uint16_t*>(k_cache),
                        static_cast<const uint16_t*>(v_cache), t0, nt, g, w);
        else
          attn_task_f32(a, static_cast<const float*>(k_cache), static_cast<const float*>(v_cache),
                        t0, nt, g, w);
      }
  }
  return 0;
}

}  // namespace swarm_native

namespace swarm_native {

// One value head's recurrence over the T rows (per-ISA clones; the OpenMP
// loop over heads stays outside them).
SWARM_CLONES static void delta_head(const float* q, const float* k, const float* v,
                                    const float* g, const float* beta, float* state, float* out,
                                    int T, int nk, int nv, int dk, int dv, int h, float* kv,
                                    float* d) {
  const int rep = nv / nk;
  float* S = state + (size_t)h * dk * dv;
  const int kh = h / rep;
  for (int t = 0; t < T; ++t) {
    const float* kt = k + ((size_t)t * nk + kh) * dk;
    const float* qt = q + ((size_t)t * nk + kh) * dk;
    const float* vt = v + ((size_t)t * nv + h) * dv;
    const float decay = exp_fast(g[(size_t)t * nv + h]);
    const float b = beta[(size_t)t * nv + h];
    for (int j = 0; j < dv; ++j) kv[j] = 0.f;
    for (int i = 0; i < dk; ++i) {  // decay the state and read it at k in one pass
      float* Si = S + (size_t)i * dv;
      const float ki = kt[i];
#pragma omp simd
      for (int j = 0; j < dv; ++j) {
        Si[j] *= decay;
        kv[j] += Si[j] * ki;
      }
    }
#pragma omp simd
    for (int j = 0; j < dv; ++j) d[j] = b * (vt[j] - kv[j]);
    float* o = out + ((size_t)t * nv + h) * dv;
    for (int j = 0; j < dv; ++j) o[j] = 0.f;
    for (int i = 0; i < dk; ++i) {  // rank-1 update, then read at q
      float* Si = S + (size_t)i * dv;
      const float ki = kt[i], qi = qt[i];
#pragma omp simd
      for (int j = 0; j < dv; ++j) {
        Si[j] += ki * d[j];
        o[j] += Si[j] * qi;
      }
    }
  }
}

void cpu_delta_rule(const float* q, const float* k, const float* v, const float* g,
                    const float* beta, float* state, float* out, int T, int nk, int nv, int dk,
                    int dv) {
#pragma omp parallel
  {
    std::vector<float> kv(dv), d(dv);
#pragma omp for schedule(static)
    for (int h = 0; h < nv; ++h)
      delta_head(q, k, v, g, beta, state, out, T, nk, nv, dk, dv, h, kv.data(), d.data());
  }
}

}  // namespace swarm_native
