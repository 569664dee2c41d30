// Paged attention and the SwiGLU tail on the host CPU.
//
// cpu_paged_attention: every (token, KV head) pair is one OpenMP task that
// serves all the query heads sharing that KV head, so a key/value row is
// converted to fp32 once per group, not once per query head.  Keys are
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

#include <cmath>
#include <cstring>
#include <vector>

namespace swarm_native {
namespace {

constexpr int kChunk = 256;

// fp16 -> fp32 without branches, so a row converts in vector registers: the
// 15 magnitude bits moved to the float's exponent/mantissa position are the
// value times 2^-112 (subnormal halves land on float subnormals, exactly),
// so one multiply by 2^112 rescales; exponent 31 (inf / NaN) is patched.
inline float half_to_float(uint16_t h) {
  const uint32_t mag = (uint32_t)(h & 0x7FFF) << 13;
  float f;
  std::memcpy(&f, &mag, 4);
  f *= 5.192296858534828e33f;  // 2^112
  uint32_t bits;
  std::memcpy(&bits, &f, 4);
  if ((h & 0x7C00) == 0x7C00) bits = 0x7F800000u | mag;  // inf / NaN keep their payload
  bits |= (uint32_t)(h & 0x8000) << 16;
  std::memcpy(&f, &bits, 4);
  return f;
}

}  // namespace

float exp_approx(float x) {
  // n = round(x / ln2), r = x - n ln2 with ln2 split into a high part with a
  // short mantissa (n * hi is exact) and the remainder (Cody and Waite), so r
  // keeps full precision however large n is; e^x = 2^n e^r, |r| <= ln2 / 2.
  if (x < -87.3f) return 0.f;
  if (x > 88.7f) x = 88.7f;
  const float n = std::nearbyint(x * 1.44269504088896341f);
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
  return p * s;
}

void cpu_silu_mul(const float* g, const float* u, float* out, int64_t n, float limit, float alpha) {
#pragma omp parallel for simd schedule(static) if (n > 65536)
  for (int64_t i = 0; i < n; ++i) {
    float a = g[i], b = u[i];
    if (limit > 0.f) {  // gpt-oss: clamped gate, clamped and shifted up, sigmoid(alpha g)
      a = a < limit ? a : limit;
      b = b < -limit ? -limit : b > limit ? limit : b;
      out[i] = a / (1.f + exp_approx(-alpha * a)) * (b + 1.f);
    } else {
      out[i] = a / (1.f + exp_approx(-a)) * b;
    }
  }
}

template <typename KV>
static inline float kv_load(const KV* p, int i);
template <>
inline float kv_load<float>(const float* p, int i) {
  return p[i];
}
template <>
inline float kv_load<uint16_t>(const uint16_t* p, int i) {
  return half_to_float(p[i]);
}

template <typename KV>
static void attention_t(const AttnArgs& a, const KV* kc, const KV* vc) {
  const int N = a.n_tokens, nq = a.n_heads, nkv = a.n_kv_heads, d = a.head_dim;
  const int rep = nq / nkv, ps = a.page_size;
#pragma omp parallel
  {
    std::vector<float> s((size_t)rep * kChunk), acc((size_t)rep * d), krow(d), vrow(d);
    std::vector<float> m(rep), l(rep);
#pragma omp for collapse(2) schedule(dynamic)
    for (int t = 0; t < N; ++t)
      for (int g = 0; g < nkv; ++g) {
        const int Lt = a.seq_lens[t];
        const int lo = a.window > 0 && Lt > a.window ? Lt - a.window : 0;
        const float* q = a.q + ((size_t)t * nq + (size_t)g * rep) * d;
        const int32_t* bt = a.block_table + (size_t)t * a.max_pages;
        const int ts = a.tree_start ? a.tree_start[t] : 0;
        const uint64_t tm = a.tree_mask ? (uint64_t)a.tree_mask[t] : 0;
        std::fill(acc.begin(), acc.end(), 0.f);
        std::fill(m.begin(), m.end(), -INFINITY);
        std::fill(l.begin(), l.end(), 0.f);
        for (int c0 = lo; c0 < Lt; c0 += kChunk) {
          const int nc = Lt - c0 < kChunk ? Lt - c0 : kChunk;
          for (int j = 0; j < nc; ++j) {
            const int key = c0 + j;
            bool vis = true;
            if (a.tree_mask) {
              const int rel = key - ts;
              vis = rel < 0 || (rel < 64 && ((tm >> rel) & 1));
            }
            if (!vis) {
              for (int h = 0; h < rep; ++h) s[(size_t)h * kChunk + j] = -INFINITY;
              continue;
            }
            const size_t off =
                (((size_t)bt[key / ps] * nkv + g) * ps + (size_t)(key % ps)) * (size_t)d;
            for (int i = 0; i < d; ++i) krow[i] = kv_load(kc + off, i);
            for (int h = 0; h < rep; ++h) {
              const float* qh = q + (size_t)h * d;
              float dot = 0.f;
#pragma omp simd reduction(+ : dot)
              for (int i = 0; i < d; ++i) dot += qh[i] * krow[i];
              dot *= a.scale;
              if (a.softcap > 0.f) dot = a.softcap * std::tanh(dot / a.softcap);
              s[(size_t)h * kChunk + j] = dot;
            }
          }
          for (int h = 0; h < rep; ++h) {
            float* sh = s.data() + (size_t)h * kChunk;
            float mx = m[h];
            for (int j = 0; j < nc; ++j) mx = sh[j] > mx ? sh[j] : mx;
            if (mx == -INFINITY) continue;  // nothing visible yet
            const float corr = m[h] == -INFINITY ? 0.f : exp_approx(m[h] - mx);
            float sum = 0.f;
#pragma omp simd reduction(+ : sum)
            for (int j = 0; j < nc; ++j) {
              const float p = sh[j] == -INFINITY ? 0.f : exp_approx(sh[j] - mx);
              sh[j] = p;
              sum += p;
            }
            l[h] = l[h] * corr + sum;
            m[h] = mx;
            float* ah = acc.data() + (size_t)h * d;
            for (int i = 0; i < d; ++i) ah[i] *= corr;
          }
          for (int j = 0; j < nc; ++j) {
            const int key = c0 + j;
            const size_t off =
                (((size_t)bt[key / ps] * nkv + g) * ps + (size_t)(key % ps)) * (size_t)d;
            bool any = false;
            for (int h = 0; h < rep; ++h) any |= s[(size_t)h * kChunk + j] > 0.f;
            if (!any) continue;
            for (int i = 0; i < d; ++i) vrow[i] = kv_load(vc + off, i);
            for (int h = 0; h < rep; ++h) {
              const float p = s[(size_t)h * kChunk + j];
              if (p == 0.f) continue;
              float* ah = acc.data() + (size_t)h * d;
#pragma omp simd
              for (int i = 0; i < d; ++i) ah[i] += p * vrow[i];
            }
          }
        }
        for (int h = 0; h < rep; ++h) {
          float den = l[h], sc = 1.f;
          if (a.sinks) {
            const float sk = a.sinks[g * rep + h];
            const float mx = m[h] > sk ? m[h] : sk;
            sc = m[h] == -INFINITY ? 0.f : exp_approx(m[h] - mx);
            den = l[h] * sc + exp_approx(sk - mx);
          }
          const float inv = den > 0.f ? sc / den : 0.f;
          float* o = a.out + ((size_t)t * nq + (size_t)g * rep + h) * d;
          const float* ah = acc.data() + (size_t)h * d;
          for (int i = 0; i < d; ++i) o[i] = ah[i] * inv;
        }
      }
  }
}

int cpu_paged_attention(const AttnArgs& a, const void* k_cache, const void* v_cache,
                        bool kv_fp16) {
  if (a.n_heads % a.n_kv_heads != 0 || a.head_dim <= 0 || a.page_size <= 0) return -1;
  if (kv_fp16)
    attention_t(a, static_cast<const uint16_t*>(k_cache), static_cast<const uint16_t*>(v_cache));
  else
    attention_t(a, static_cast<const float*>(k_cache), static_cast<const float*>(v_cache));
  return 0;
}

}  // namespace swarm_native

namespace swarm_native {

void cpu_delta_rule(const float* q, const float* k, const float* v, const float* g,
                    const float* beta, float* state, float* out, int T, int nk, int nv, int dk,
                    int dv) {
  const int rep = nv / nk;
#pragma omp parallel for schedule(static)
  for (int h = 0; h < nv; ++h) {
    float* S = state + (size_t)h * dk * dv;
    std::vector<float> kv(dv), d(dv);
    const int kh = h / rep;
    for (int t = 0; t < T; ++t) {
      const float* kt = k + ((size_t)t * nk + kh) * dk;
      const float* qt = q + ((size_t)t * nk + kh) * dk;
      const float* vt = v + ((size_t)t * nv + h) * dv;
      const float decay = std::exp(g[(size_t)t * nv + h]);
      const float b = beta[(size_t)t * nv + h];
      std::fill(kv.begin(), kv.end(), 0.f);
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
      std::fill(o, o + dv, 0.f);
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
}

}  // namespace swarm_native
