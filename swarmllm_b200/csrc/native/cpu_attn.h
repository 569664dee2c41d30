// Paged attention, SwiGLU tail and exp on the host CPU.
#pragma once
#include <cstdint>

namespace swarm_native {

struct AttnArgs {
  const float* q;             // [n_tokens, n_heads, head_dim], rotated
  float* out;                 // [n_tokens, n_heads, head_dim]
  const int32_t* block_table; // [n_tokens, max_pages]
  const int32_t* seq_lens;    // [n_tokens]: keys 0..seq_len-1 are attended
  const int32_t* tree_start;  // [n_tokens] or null: first key of the draft tree
  const int64_t* tree_mask;   // [n_tokens] or null: bit r = tree key tree_start + r visible
  const float* sinks;         // [n_heads] or null: per-head sink logit
  int n_tokens, n_heads, n_kv_heads, head_dim, page_size, max_pages;
  int window;                 // > 0: only the last `window` keys
  float scale, softcap;       // softcap > 0: s = c tanh(s / c)
};

// K / V caches [pages, n_kv_heads, page_size, head_dim], fp16 or fp32.
int cpu_paged_attention(const AttnArgs& a, const void* k_cache, const void* v_cache, bool kv_fp16);

// out = silu(g) * u, or with limit > 0 the clamped gpt-oss form
// min(g, limit) * sigmoid(alpha min(g, limit)) * (clamp(u, +-limit) + 1).
void cpu_silu_mul(const float* g, const float* u, float* out, int64_t n, float limit, float alpha);

// e^x as 2^n e^r, |r| <= ln2 / 2 (Cody-Waite reduction), e^r by its degree-6
// Taylor polynomial; 0 below -87.3, clamped at 88.7.
float exp_approx(float x);

}  // namespace swarm_native

namespace swarm_native {

// Gated delta rule over one sequence's rows, per value head h (OpenMP over
// heads), state S [nv][dk][dv] fp32 updated in place:
//   S = exp(g[t,h]) S;  d = beta[t,h] (v_t - S^T k_t);  S += k_t d^T;  o_t = S^T q_t
// q, k [T][nk][dk] (value head h reads key head h / (nv / nk)), v, out
// [T][nv][dv], g, beta [T][nv].
void cpu_delta_rule(const float* q, const float* k, const float* v, const float* g,
                    const float* beta, float* state, float* out, int T, int nk, int nv, int dk,
                    int dv);

}  // namespace swarm_native
