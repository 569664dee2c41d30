// Diagnostics: the issue rate of tcgen05.mma kind::f16 shapes.
//
// One CTA per SM issues `iters` x 4 MMAs of one shape (M x N x 16, fp16 in,
// fp32 accumulate) back to back from one thread, commits once and waits; the
// clock64 difference per MMA is what a weight-streaming GEMM pays per
// instruction.  With `group` > 0 the thread commits after every `group` MMAs
// (mode bit 0: and waits for completion -- the round trip a pipeline pays when
// it has to see MMAs finish before it can refill their operands; bit 1: the
// MMAs rotate over 4 accumulators; bit 2: instead of committing, the thread
// spins `spin` clocks, idling the issue like a wait would).  Operands are
// whatever shared memory / TMEM holds (the values do not matter), laid out
// as the GEMMs lay theirs out: K-major, 128-byte
// swizzle, 8-row groups of 1024 bytes, four K = 16 steps inside one 128-byte
// row.  TS = A from TMEM (the quantized GEMM's form), SS = A from shared memory.
#include "kernels.h"

#include "common.cuh"
#include "tc_utils.cuh"

namespace swarm {
using namespace tc;

template <bool TS, int M, int N>
struct ProbeCfg {
  static constexpr int A_BYTES = TS ? 0 : M * 128;
  static constexpr int B_BYTES = N * 128;
  static constexpr int SMEM = 1024 + A_BYTES + B_BYTES + 64;
  // D accumulators (4 for the rotating mode, which needs 4N + 32 <= 512) + A for TS
  static constexpr bool ROT_OK = 4 * N + 32 <= 512;
  static constexpr int NEED = (ROT_OK ? 4 * N : N) + (TS ? 32 : 0);
  static constexpr int COLS = NEED <= 32 ? 32 : NEED <= 64 ? 64 : NEED <= 128 ? 128
                              : NEED <= 256 ? 256 : 512;
};

template <bool TS, int M, int N>
__global__ void __launch_bounds__(128, 1) mma_probe_kernel(int iters, int group, int mode,
                                                           int spin, long long* cycles) {
  using P = ProbeCfg<TS, M, N>;
  extern __shared__ __align__(1024) uint8_t probe_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(probe_raw) + 1023) &
                                           ~uintptr_t(1023));
  uint8_t* a_s = sm;
  uint8_t* b_s = sm + P::A_BYTES;
  uint64_t* bar = reinterpret_cast<uint64_t*>(b_s + P::B_BYTES);
  uint32_t* slot = reinterpret_cast<uint32_t*>(bar + 1);
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(slot, P::COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t base = *slot;
  if (threadIdx.x == 0) {
    const uint32_t idesc = idesc_f16(M, N, 0);
    const uint64_t adesc = smem_desc(smem_u32(a_s), 16, 1024, 2);
    const uint64_t bdesc = smem_desc(smem_u32(b_s), 16, 1024, 2);
    const long long t0 = clock64();
    uint32_t phase = 0;
    int issued = 0;
    const bool rotate = P::ROT_OK && (mode & 2) != 0;
    const uint32_t a_col = (uint32_t)((P::ROT_OK ? 4 : 1) * N);   // A (TS) after the D columns
    for (int it = 0; it < iters; ++it) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint32_t d = base + (rotate ? (uint32_t)(kk * N) : 0u);
        if constexpr (TS)
          umma_f16_ts(d, base + a_col + kk * 8, bdesc + (uint64_t)((kk * 32) >> 4), idesc, 1u);
        else
          umma_f16_ss(d, adesc + (uint64_t)((kk * 32) >> 4),
                      bdesc + (uint64_t)((kk * 32) >> 4), idesc, 1u);
      }
      issued += 4;
      if (group > 0 && issued % group == 0) {
        if (mode & 4) {
          const long long ts = clock64();
          while (clock64() - ts < spin) {
          }
        } else {
          umma_commit(bar);
          if (mode & 1) {
            if (!mbar_wait(bar, phase, nullptr, 0)) break;
            phase ^= 1;
          }
        }
      }
    }
    if (group > 0 && !(mode & 1) && !(mode & 4)) {
      // commits without waits: their arrivals completed phases in passing;
      // count them to know the parity of the final one
      phase = (uint32_t)((issued / group) & 1);
    }
    umma_commit(bar);
    mbar_wait(bar, phase, nullptr, 0);
    cycles[blockIdx.x] = clock64() - t0;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(base, P::COLS);
}

template <bool TS, int M, int N>
static int probe_t(int iters, int group, int mode, int spin, int ctas, long long* cycles,
                   cudaStream_t s) {
  using P = ProbeCfg<TS, M, N>;
  static_assert(P::NEED <= 512, "TMEM columns");
  if ((mode & 2) && !P::ROT_OK) return -1;
  static unsigned long long done = 0;
  if (!smem_attr_once(mma_probe_kernel<TS, M, N>, P::SMEM, &done)) return -3;
  mma_probe_kernel<TS, M, N><<<ctas, 128, P::SMEM, s>>>(iters, group, mode, spin, cycles);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}

}  // namespace swarm

using namespace swarm;

// Shapes, by index: the (TS?, M, N) of mma_probe_shape().
static const int kProbeShapes[][3] = {
    {1, 128, 16}, {1, 128, 32}, {1, 128, 64}, {1, 128, 128}, {1, 128, 256},
    {0, 128, 32}, {0, 128, 128}, {0, 128, 256}, {0, 64, 64}, {0, 64, 128}, {0, 64, 256}};

int mma_probe_shapes() { return (int)(sizeof(kProbeShapes) / sizeof(kProbeShapes[0])); }

void mma_probe_shape(int i, int* ts, int* m, int* n) {
  *ts = kProbeShapes[i][0];
  *m = kProbeShapes[i][1];
  *n = kProbeShapes[i][2];
}

int launch_mma_probe(int shape, int iters, int group, int mode, int spin, int ctas,
                     long long* cycles, cudaStream_t s) {
  if (group < 0 || group % 4) return -1;
  switch (shape) {
    case 0: return probe_t<true, 128, 16>(iters, group, mode, spin, ctas, cycles, s);
    case 1: return probe_t<true, 128, 32>(iters, group, mode, spin, ctas, cycles, s);
    case 2: return probe_t<true, 128, 64>(iters, group, mode, spin, ctas, cycles, s);
    case 3: return probe_t<true, 128, 128>(iters, group, mode, spin, ctas, cycles, s);
    case 4: return probe_t<true, 128, 256>(iters, group, mode, spin, ctas, cycles, s);
    case 5: return probe_t<false, 128, 32>(iters, group, mode, spin, ctas, cycles, s);
    case 6: return probe_t<false, 128, 128>(iters, group, mode, spin, ctas, cycles, s);
    case 7: return probe_t<false, 128, 256>(iters, group, mode, spin, ctas, cycles, s);
    case 8: return probe_t<false, 64, 64>(iters, group, mode, spin, ctas, cycles, s);
    case 9: return probe_t<false, 64, 128>(iters, group, mode, spin, ctas, cycles, s);
    case 10: return probe_t<false, 64, 256>(iters, group, mode, spin, ctas, cycles, s);
    default: return -1;
  }
}
