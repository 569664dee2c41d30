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
// mode 0 is a plain dense [T][rows] fp32 buffer (SIMT GEMM, tests).
// n_src > 1: the partials of n_src ranks of a tensor-parallel group, pushed
// into this rank's buffer by their GEMM epilogues, sit src_stride floats
// apart; get() then also sums over the ranks (the all-reduce happens while
// reading).
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

#ifdef __CUDACC__
  __device__ __forceinline__ float get(int t, int r) const {
    const float extra = add ? add[(size_t)t * add_stride + r] : 0.f;
    if (mode == 0) return ws[(size_t)t * rows + r] + extra;
    const int rt = r >> 7, rr = r & 127;
    const int nt = t / tok_tile, tt = t - nt * tok_tile;
    const int tile = rt * n_tok_tiles + nt;
    const long u0 = (long)tile * ksb;
    const int c0 = (int)(u0 / upc);
    const int c1 = (int)((u0 + ksb - 1) / upc);
    float acc = extra;
    const int ns = n_src > 1 ? n_src : 1;
    for (int s = 0; s < ns; ++s) {
      const float* w = ws + (size_t)s * src_stride;
      for (int c = c0; c <= c1; ++c) acc += w[((size_t)(tile + c) * tok_tile + tt) * 128 + rr];
    }
    return acc;
  }
#endif
};

}  // namespace swarm
