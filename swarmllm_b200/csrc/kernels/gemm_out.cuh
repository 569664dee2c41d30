// GemmOut: how an epilogue kernel reads the fp32 result of a quantized GEMM.
//
// The tensor-core GEMM (qgemm_tc.cu) is persistent and stream-K balanced: the
// (row-tile x token-tile x k-unit) work is cut into equal contiguous ranges,
// one per CTA, so a tile's K reduction can be split over a few CTAs.  Each CTA
// writes its partial accumulator for a tile into slot (tile + cta) of a
// workspace laid out [slot][tok_tile][128] fp32 (the slot is unique because
// CTAs cover consecutive unit ranges).  Instead of a separate reduction pass,
// every epilogue kernel (RoPE + KV append, residual + RMSNorm, SwiGLU, logits
// copy) sums the segments while it reads, which saves one write + read of the
// [T, rows] result.
//
// mode 0 is a plain dense [T][rows] fp32 buffer (SIMT GEMM, tests, the MoE
// combine's per-rank partials under tensor parallelism).
// n_src > 1 (either mode): the partials of n_src ranks of a tensor-parallel
// group, stored into this rank's buffer by their epilogues, sit src_stride
// floats apart; get() then also sums over the ranks (the reduction happens
// while reading).
// The struct is plain data so host C++ (the torch bindings) can hold it.
#pragma once
#include <stddef.h>

namespace swarm {

struct GemmOut {
  const float* ws;
  int rows;       // logical output features
  int T;          // tokens
  int mode;       // 0 dense, 1 stream-K tiles
  int ksb;        // k-units per tile
  int upc;        // k-units per CTA
  int tok_tile;   // tokens per token-tile (N of the MMA)
  int n_tok_tiles;
  int seg_max;    // unused; kept so the struct layout stays fixed
  int n_src;      // ranks whose partials are summed (0 or 1: just this one)
  long long src_stride;
  const float* add;  // optional dense [T][add_stride] term added on read (LoRA deltas)
  int add_stride;
  // set by gemm_out_finalize(): every element read divides by neither
  int tok_shift;     // log2(tok_tile)
  float inv_upc;     // 1 / upc

#ifdef __CUDACC__
  // floor(u / upc) from a float estimate, corrected to the exact quotient
  // (u < 2^24 keeps the estimate within one).
  __device__ __forceinline__ int cta_of(int u) const {
    int c = __float2int_rz((float)u * inv_upc);
    if (c * upc > u) --c;
    else if ((c + 1) * upc <= u) ++c;
    return c;
  }

  __device__ __forceinline__ float get(int t, int r) const {
    const float extra = add ? add[(size_t)t * add_stride + r] : 0.f;
    if (mode == 0) {
      float acc = extra;
      const int ns = n_src > 1 ? n_src : 1;
      for (int s = 0; s < ns; ++s) acc += ws[(size_t)s * src_stride + (size_t)t * rows + r];
      return acc;
    }
    const int rt = r >> 7, rr = r & 127;
    const int nt = t >> tok_shift, tt = t & (tok_tile - 1);
    const int tile = rt * n_tok_tiles + nt;
    const int u0 = tile * ksb;
    const int c0 = cta_of(u0);
    const int c1 = cta_of(u0 + ksb - 1);
    float acc = extra;
    const int ns = n_src > 1 ? n_src : 1;
    for (int s = 0; s < ns; ++s) {
      const float* w = ws + (size_t)s * src_stride;
      for (int c = c0; c <= c1; ++c) acc += w[((size_t)(tile + c) * tok_tile + tt) * 128 + rr];
    }
    return acc;
  }

  // Rows r..r+3 (r % 4 == 0) with 16-byte loads: four rows of one 128-row
  // group are contiguous in every slot.  Needs rows % 4 == 0 (mode 0) and
  // 16-byte aligned partial buffers (workspaces are).
  __device__ __forceinline__ float4 get4(int t, int r) const {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (add) {
      const float* a = add + (size_t)t * add_stride + r;
      acc = make_float4(a[0], a[1], a[2], a[3]);
    }
    if (mode == 0) {
      const int ns = n_src > 1 ? n_src : 1;
      for (int s = 0; s < ns; ++s) {
        const float4 v =
            *reinterpret_cast<const float4*>(ws + (size_t)s * src_stride + (size_t)t * rows + r);
        acc = make_float4(acc.x + v.x, acc.y + v.y, acc.z + v.z, acc.w + v.w);
      }
      return acc;
    }
    const int rt = r >> 7, rr = r & 127;
    const int nt = t >> tok_shift, tt = t & (tok_tile - 1);
    const int tile = rt * n_tok_tiles + nt;
    const int u0 = tile * ksb;
    const int c0 = cta_of(u0);
    const int c1 = cta_of(u0 + ksb - 1);
    const int ns = n_src > 1 ? n_src : 1;
    for (int s = 0; s < ns; ++s) {
      const float* w = ws + (size_t)s * src_stride;
      for (int c = c0; c <= c1; ++c) {
        const float4 v =
            *reinterpret_cast<const float4*>(w + ((size_t)(tile + c) * tok_tile + tt) * 128 + rr);
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
    }
    return acc;
  }

  // Rows r .. r + 7 of token t (r a multiple of 8: one 128-row tile, so one
  // segment lookup serves all eight).
  __device__ __forceinline__ void get8(int t, int r, float4& lo, float4& hi) const {
    lo = make_float4(0.f, 0.f, 0.f, 0.f);
    hi = lo;
    if (add) {
      const float* a = add + (size_t)t * add_stride + r;
      lo = make_float4(a[0], a[1], a[2], a[3]);
      hi = make_float4(a[4], a[5], a[6], a[7]);
    }
    const float* base;
    if (mode == 0) {
      const int ns = n_src > 1 ? n_src : 1;
      for (int s = 0; s < ns; ++s) {
        base = ws + (size_t)s * src_stride + (size_t)t * rows + r;
        const float4 v0 = *reinterpret_cast<const float4*>(base);
        const float4 v1 = *reinterpret_cast<const float4*>(base + 4);
        lo = make_float4(lo.x + v0.x, lo.y + v0.y, lo.z + v0.z, lo.w + v0.w);
        hi = make_float4(hi.x + v1.x, hi.y + v1.y, hi.z + v1.z, hi.w + v1.w);
      }
      return;
    }
    const int rt = r >> 7, rr = r & 127;
    const int nt = t >> tok_shift, tt = t & (tok_tile - 1);
    const int tile = rt * n_tok_tiles + nt;
    const int u0 = tile * ksb;
    const int c0 = cta_of(u0);
    const int c1 = cta_of(u0 + ksb - 1);
    const int ns = n_src > 1 ? n_src : 1;
    for (int s = 0; s < ns; ++s) {
      const float* w = ws + (size_t)s * src_stride;
      for (int c = c0; c <= c1; ++c) {
        const float* p = w + ((size_t)(tile + c) * tok_tile + tt) * 128 + rr;
        const float4 v0 = *reinterpret_cast<const float4*>(p);
        const float4 v1 = *reinterpret_cast<const float4*>(p + 4);
        lo.x += v0.x; lo.y += v0.y; lo.z += v0.z; lo.w += v0.w;
        hi.x += v1.x; hi.y += v1.y; hi.z += v1.z; hi.w += v1.w;
      }
    }
  }
#endif
};

// Fill the derived fields of a stream-K GemmOut (host side, after tok_tile /
// upc are set).  tok_tile is a power of two; unit counts stay below 2^24.
inline void gemm_out_finalize(GemmOut* g) {
  int s = 0;
  while ((1 << s) < g->tok_tile) ++s;
  g->tok_shift = s;
  g->inv_upc = g->upc > 0 ? 1.0f / (float)g->upc : 0.f;
}

}  // namespace swarm
