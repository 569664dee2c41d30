// Token selection on the device: greedy argmax and temperature / top-k /
// top-p sampling by the Gumbel-max trick with counter-based noise.
//
// The noise for (seed, position, token) comes from Philox4x32-10 (Salmon et
// al., "Parallel Random Numbers: As Easy as 1, 2, 3", SC'11), so any rank or a
// drafter that knows the seed and position redraws exactly the same Gumbel
// variates: this is what makes coupled speculative sampling reproducible across
// GPUs (the reference does the same on the host with Philox4x64-10,
// src/inference/coupled_noise.rs:39,61).
//
// Top-k: the k-th largest logit is found by a 4-pass radix select over the
// order-preserving integer image of the floats.  Top-p: the probability
// threshold is found by bisection on the sorted-free "mass above tau" count.
// Tokens below either threshold get no Gumbel draw.
#include "kernels.h"
#include "common.cuh"

namespace swarm {

SW_DEVICE uint32_t mulhilo(uint32_t a, uint32_t b, uint32_t& hi) {
  hi = __umulhi(a, b);
  return a * b;
}

// Philox4x32 with 10 rounds.
SW_DEVICE uint4 philox4x32_10(uint4 ctr, uint2 key) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u, W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    uint32_t hi0, hi1;
    uint32_t lo0 = mulhilo(M0, ctr.x, hi0);
    uint32_t lo1 = mulhilo(M1, ctr.z, hi1);
    ctr = make_uint4(hi1 ^ ctr.y ^ key.x, lo1, hi0 ^ ctr.w ^ key.y, lo0);
    key.x += W0;
    key.y += W1;
  }
  return ctr;
}

// Uniform in (0,1) for (seed, position, token).
SW_DEVICE float philox_uniform(uint64_t seed, uint32_t position, uint32_t token) {
  uint4 c = make_uint4(token, position, 0x5eedu, 0u);
  uint2 k = make_uint2((uint32_t)seed, (uint32_t)(seed >> 32));
  uint4 r = philox4x32_10(c, k);
  // 24 random bits -> (0,1), never 0 or 1.
  return ((r.x >> 8) + 0.5f) * (1.0f / 16777216.0f);
}

SW_DEVICE uint32_t float_key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

struct ArgMax {
  float v;
  int i;
};

SW_DEVICE ArgMax argmax_merge(ArgMax a, ArgMax b) {
  if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
  return a;
}

SW_DEVICE ArgMax block_argmax(ArgMax x, float* sv, int* si) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ArgMax y{__shfl_xor_sync(0xffffffffu, x.v, o), __shfl_xor_sync(0xffffffffu, x.i, o)};
    x = argmax_merge(x, y);
  }
  __syncthreads();
  if (lane == 0) { sv[wid] = x.v; si[wid] = x.i; }
  __syncthreads();
  if (wid == 0) {
    ArgMax y = (lane < nw) ? ArgMax{sv[lane], si[lane]} : ArgMax{-INFINITY, 0x7fffffff};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      ArgMax z{__shfl_xor_sync(0xffffffffu, y.v, o), __shfl_xor_sync(0xffffffffu, y.i, o)};
      y = argmax_merge(y, z);
    }
    if (lane == 0) { sv[0] = y.v; si[0] = y.i; }
  }
  __syncthreads();
  return ArgMax{sv[0], si[0]};
}

// Split argmax for few rows over a large vocabulary: a grid of (row, slice)
// CTAs each merge their slice's winner into one 64-bit key per row with
// atomicMax -- order-preserving image of the float in the high word, the
// complemented index in the low word (ties -> lower index) -- and a second
// kernel unpacks it and clears the key for the next use.
constexpr int kArgmaxMaxRows = 4096;
__device__ unsigned long long g_argmax_keys[kArgmaxMaxRows];

SW_DEVICE uint32_t float_order_bits(float v) {
  const uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__global__ void __launch_bounds__(256) argmax_split_kernel(const float* __restrict__ logits, int V,
                                                           int stride, int slice) {
  __shared__ float sv[32];
  __shared__ int si[32];
  const int row = blockIdx.x;
  const float* r = logits + (size_t)row * stride;
  const int lo = blockIdx.y * slice, hi = min(V, lo + slice);
  ArgMax best{-INFINITY, 0x7fffffff};
  for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) best = argmax_merge(best, ArgMax{r[i], i});
  best = block_argmax(best, sv, si);
  if (threadIdx.x == 0 && best.i != 0x7fffffff) {
    const unsigned long long key = ((unsigned long long)float_order_bits(best.v) << 32) |
                                   (unsigned long long)(0xFFFFFFFFu - (uint32_t)best.i);
    atomicMax(&g_argmax_keys[row], key);
  }
}

__global__ void argmax_finish_kernel(int rows, int32_t* __restrict__ out, float* __restrict__ out_val) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  const unsigned long long key = g_argmax_keys[row];
  g_argmax_keys[row] = 0ull;
  out[row] = (int32_t)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
  if (out_val) {
    const uint32_t hb = (uint32_t)(key >> 32);
    out_val[row] = __uint_as_float((hb & 0x80000000u) ? (hb & 0x7FFFFFFFu) : ~hb);
  }
}

__global__ void __launch_bounds__(1024) argmax_kernel(const float* __restrict__ logits, int V,
                                                      int stride, int32_t* __restrict__ out,
                                                      float* __restrict__ out_val) {
  __shared__ float sv[32];
  __shared__ int si[32];
  const float* row = logits + (size_t)blockIdx.x * stride;
  ArgMax best{-INFINITY, 0x7fffffff};
  for (int i = threadIdx.x; i < V; i += blockDim.x) best = argmax_merge(best, ArgMax{row[i], i});
  best = block_argmax(best, sv, si);
  if (threadIdx.x == 0) {
    out[blockIdx.x] = best.i;
    if (out_val) out_val[blockIdx.x] = best.v;
  }
}

// ---- temperature / top-k / top-p sampling -------------------------------------
//
// Semantics (mirrored by the host sampler): keep the tokens whose logit is >=
// the k-th largest (ties kept); over those, probabilities softmax((l - max) / T);
// keep the smallest most-probable set whose mass reaches top_p, plus every token
// tied with its last member; draw by Gumbel-max with Philox noise per
// (seed, position, token).
//
// Two paths, one CTA per row:
//  * top-k of at most kSampleCand tokens: radix select of the k-th key (4
//    passes over the row, warp-aggregated counts), the survivors gathered into
//    shared memory and bitonic-sorted, and the top-p cut and the draw done on
//    that short list;
//  * otherwise: radix select of the top-p cut directly on probability mass
//    (64-bit fixed point, so the shared-memory sums are order-independent and
//    reruns bit-identical), then one pass drawing over the survivors.
constexpr int kSampleCand = 2048;
constexpr double kMassOne = 1099511627776.0;   // 2^40: fixed-point unit of probability mass

// Largest key T with weight(key >= T) >= want among keys >= floor_key; weight 1
// per token (MASS = false) or its fixed-point probability.
template <bool MASS>
SW_DEVICE uint32_t radix_select(const float* __restrict__ row, int V, uint32_t floor_key,
                                unsigned long long want, float mx, float inv_t, float inv_z,
                                unsigned long long* hist, uint32_t* prefix_s,
                                unsigned long long* want_s) {
  if (threadIdx.x == 0) { *prefix_s = 0; *want_s = want; }
  const int lane = threadIdx.x & 31;
  uint32_t mask = 0;
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int b = threadIdx.x; b < 256; b += blockDim.x) hist[b] = 0;
    __syncthreads();
    const uint32_t prefix = *prefix_s;
    // four loads in flight per thread; uniform trip count per warp (the warp
    // intrinsics below need every lane)
    for (int base = 0; base < V; base += 4 * blockDim.x) {
      float l[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = base + u * blockDim.x + threadIdx.x;
        l[u] = i < V ? row[i] : 0.f;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = base + u * blockDim.x + threadIdx.x;
        int bin = -1;
        if (i < V) {
          const uint32_t key = float_key(l[u]);
          if (key >= floor_key && (key & mask) == prefix) bin = (int)((key >> shift) & 255u);
        }
        if (!__any_sync(0xffffffffu, bin >= 0)) continue;   // warp-uniform: later passes skip most
        const unsigned same = __match_any_sync(0xffffffffu, bin);
        const bool leader = lane == __ffs(same) - 1;
        if (MASS) {
          // exact group sum of the 40-bit weights as two 20-bit halves (each < 2^25)
          const unsigned long long w =
              bin >= 0 ? (unsigned long long)((double)(expf((l[u] - mx) * inv_t) * inv_z) * kMassOne)
                       : 0ull;
          const unsigned lo = __reduce_add_sync(same, (unsigned)(w & 0xFFFFFull));
          const unsigned hi = __reduce_add_sync(same, (unsigned)(w >> 20));
          if (bin >= 0 && leader) atomicAdd(&hist[bin], ((unsigned long long)hi << 20) + lo);
        } else {
          if (bin >= 0 && leader) atomicAdd(&hist[bin], (unsigned long long)__popc(same));
        }
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      const unsigned long long need = *want_s;
      unsigned long long acc = 0;
      int b = 255;
      for (; b > 0; --b) {
        if (acc + hist[b] >= need) break;
        acc += hist[b];
      }
      *want_s = need - acc;
      *prefix_s = prefix | ((uint32_t)b << shift);
    }
    mask |= 255u << shift;
    __syncthreads();
  }
  return *prefix_s;
}

__global__ void __launch_bounds__(1024, 1) sample_kernel(
    const float* __restrict__ logits, int V, int stride, const float* __restrict__ temperature,
    const int32_t* __restrict__ top_k, const float* __restrict__ top_p,
    const uint64_t* __restrict__ seeds, const int32_t* __restrict__ positions,
    int32_t* __restrict__ out) {
  __shared__ float sv[32];
  __shared__ int si[32];
  __shared__ float red[32];
  __shared__ unsigned long long hist[256];
  __shared__ uint32_t prefix_s;
  __shared__ unsigned long long want_s;
  __shared__ unsigned long long cand[kSampleCand];   // (key << 32) | ~index, sorted descending
  __shared__ float cum[kSampleCand];
  __shared__ int n_s, cut_s;
  const int r = blockIdx.x;
  const float* row = logits + (size_t)r * stride;
  const float temp = temperature[r];
  ArgMax best{-INFINITY, 0x7fffffff};
  if (!(temp > 0.f)) {
    for (int i = threadIdx.x; i < V; i += blockDim.x) best = argmax_merge(best, ArgMax{row[i], i});
    best = block_argmax(best, sv, si);
    if (threadIdx.x == 0) out[r] = best.i;
    return;
  }
  const float inv_t = 1.f / temp;
  const uint64_t seed = seeds ? seeds[r] : 0ull;
  const uint32_t pos = positions ? (uint32_t)positions[r] : 0u;
  int k = top_k ? top_k[r] : 0;
  if (k >= V) k = 0;
  const float tp = top_p ? top_p[r] : 1.f;

  uint32_t floor_key = 0;   // keep keys >= floor_key
  if (k > 0) {
    floor_key = radix_select<false>(row, V, 0u, (unsigned long long)k, 0.f, 0.f, 0.f, hist,
                                    &prefix_s, &want_s);
    if (k <= kSampleCand) {
      // ---- short-list path: gather, sort, cut, draw -------------------------
      if (threadIdx.x == 0) n_s = 0;
      __syncthreads();
      for (int i = threadIdx.x; i < V; i += blockDim.x) {
        const uint32_t key = float_key(row[i]);
        if (key >= floor_key) {
          const int slot = atomicAdd(&n_s, 1);
          if (slot < kSampleCand)
            cand[slot] = ((unsigned long long)key << 32) | (uint32_t)~(uint32_t)i;
        }
      }
      __syncthreads();
      const int n = n_s;
      if (n <= kSampleCand) {   // (more only with ties at the k-th key: mass path below)
        int np2 = 1;
        while (np2 < n) np2 <<= 1;
        for (int j = n + threadIdx.x; j < np2; j += blockDim.x) cand[j] = 0ull;
        __syncthreads();
        for (int size = 2; size <= np2; size <<= 1) {           // bitonic sort, descending
          for (int stride2 = size >> 1; stride2 > 0; stride2 >>= 1) {
            for (int j = threadIdx.x; j < np2; j += blockDim.x) {
              const int o = j ^ stride2;
              if (o > j) {
                const bool desc = (j & size) == 0;
                const unsigned long long a = cand[j], b = cand[o];
                if (desc ? (a < b) : (a > b)) { cand[j] = b; cand[o] = a; }
              }
            }
            __syncthreads();
          }
        }
        const float mx = row[~(uint32_t)cand[0]];
        // probabilities (unnormalised) and their inclusive prefix sums, in sorted order
        if (threadIdx.x < 32) {
          float carry = 0.f;
          for (int c0 = 0; c0 < n; c0 += 32) {
            const int j = c0 + threadIdx.x;
            float e = j < n ? expf((row[~(uint32_t)cand[j]] - mx) * inv_t) : 0.f;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
              const float t = __shfl_up_sync(0xffffffffu, e, o);
              if ((int)threadIdx.x >= o) e += t;
            }
            if (j < n) cum[j] = carry + e;
            carry += __shfl_sync(0xffffffffu, e, 31);
          }
        }
        if (threadIdx.x == 0) cut_s = n - 1;
        __syncthreads();
        if (tp < 1.f) {
          const float want = tp * cum[n - 1];
          for (int j = threadIdx.x; j < n; j += blockDim.x)
            if (cum[j] >= want && (j == 0 || cum[j - 1] < want)) cut_s = j;
          __syncthreads();
          const uint32_t ck = (uint32_t)(cand[cut_s] >> 32);   // extend over ties
          __syncthreads();
          for (int j = threadIdx.x; j < n; j += blockDim.x)
            if ((uint32_t)(cand[j] >> 32) == ck && (j == n - 1 || (uint32_t)(cand[j + 1] >> 32) != ck))
              cut_s = j;
          __syncthreads();
        }
        const int last = cut_s;
        for (int j = threadIdx.x; j <= last; j += blockDim.x) {
          const int i = (int)~(uint32_t)cand[j];
          const float u = philox_uniform(seed, pos, (uint32_t)i);
          const float g = -logf(-logf(u));
          best = argmax_merge(best, ArgMax{(row[i] - mx) * inv_t + g, i});
        }
        best = block_argmax(best, sv, si);
        if (threadIdx.x == 0) out[r] = best.i;
        return;
      }
    }
  }
  // ---- whole-row path: top-p cut by radix select on probability mass -------
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < V; i += blockDim.x) mx = fmaxf(mx, row[i]);
  mx = block_max(mx, red);
  uint32_t cut_key = floor_key;
  if (tp < 1.f) {
    float z = 0.f;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
      const float l = row[i];
      if (float_key(l) >= floor_key) z += expf((l - mx) * inv_t);
    }
    z = block_sum(z, red);
    cut_key = radix_select<true>(row, V, floor_key, (unsigned long long)((double)tp * kMassOne), mx,
                                 inv_t, 1.f / z, hist, &prefix_s, &want_s);
  }
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float l = row[i];
    if (float_key(l) < cut_key) continue;
    const float u = philox_uniform(seed, pos, (uint32_t)i);
    const float g = -logf(-logf(u));
    best = argmax_merge(best, ArgMax{(l - mx) * inv_t + g, i});
  }
  best = block_argmax(best, sv, si);
  if (threadIdx.x == 0) out[r] = best.i;
}

// Frequency / presence penalties: row r subtracts val[i] from logit tok[i]
// for i in [off[r], off[r + 1]) -- the distinct tokens the row's request has
// generated, val = count * frequency_penalty + presence_penalty.  Tokens of a
// row are distinct, so the stores never collide.
__global__ void apply_penalties_kernel(float* __restrict__ logits, int V, int stride,
                                       const int32_t* __restrict__ off,
                                       const int32_t* __restrict__ tok,
                                       const float* __restrict__ val) {
  const int r = blockIdx.x;
  for (int i = off[r] + threadIdx.x; i < off[r + 1]; i += blockDim.x) {
    const int t = tok[i];
    if ((unsigned)t < (unsigned)V) logits[(size_t)r * stride + t] -= val[i];
  }
}

__global__ void philox_uniform_kernel(uint64_t seed, const int32_t* positions, int n_pos, int V,
                                      float* out) {
  const int r = blockIdx.y;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < V; i += gridDim.x * blockDim.x)
    out[(size_t)r * V + i] = philox_uniform(seed, (uint32_t)positions[r], (uint32_t)i);
}

}  // namespace swarm

using namespace swarm;

void launch_argmax(const float* logits, int rows, int V, int stride, int32_t* out, float* out_val,
                   cudaStream_t s) {
  if (rows <= 0) return;
  // Few rows over a big vocabulary: spread each row over ~2 waves of CTAs.
  // (The per-row keys are one static buffer: argmax launches on different
  // streams of one device must not overlap.)
  const int splits = rows >= 296 ? 1 : (296 + rows - 1) / rows;
  if (splits > 1 && V >= 8192 && rows <= kArgmaxMaxRows) {
    const int sl = ((V + splits - 1) / splits + 255) / 256 * 256;
    argmax_split_kernel<<<dim3(rows, (V + sl - 1) / sl), 256, 0, s>>>(logits, V, stride, sl);
    argmax_finish_kernel<<<(rows + 127) / 128, 128, 0, s>>>(rows, out, out_val);
  } else {
    argmax_kernel<<<rows, 1024, 0, s>>>(logits, V, stride, out, out_val);
  }
  SW_LAUNCH_CHECK();
}

void launch_sample(const float* logits, int rows, int V, int stride, const float* temperature,
                   const int32_t* top_k, const float* top_p, const uint64_t* seeds,
                   const int32_t* positions, int32_t* out, cudaStream_t s) {
  if (rows <= 0) return;
  sample_kernel<<<rows, 1024, 0, s>>>(logits, V, stride, temperature, top_k, top_p, seeds,
                                      positions, out);
  SW_LAUNCH_CHECK();
}

void launch_apply_penalties(float* logits, int rows, int V, int stride, const int32_t* off,
                            const int32_t* tok, const float* val, cudaStream_t s) {
  if (rows <= 0) return;
  apply_penalties_kernel<<<rows, 128, 0, s>>>(logits, V, stride, off, tok, val);
  SW_LAUNCH_CHECK();
}

void launch_philox_uniform(uint64_t seed, const int32_t* positions, int n_pos, int V, float* out,
                           cudaStream_t s) {
  if (n_pos <= 0) return;
  dim3 grid((V + 255) / 256 < 512 ? (V + 255) / 256 : 512, n_pos);
  philox_uniform_kernel<<<grid, 256, 0, s>>>(seed, positions, n_pos, V, out);
  SW_LAUNCH_CHECK();
}
