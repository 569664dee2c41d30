// Peer-memory signalling shared by the expert-parallel kernels (ep_comm.cu)
// and the grouped expert GEMM (moe_tc.cu).
#pragma once
#include "common.cuh"

namespace swarm {

struct EpPeers {
  unsigned long long base[8];  // arena base of every rank (own included)
};

SW_DEVICE void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
SW_DEVICE uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Raise flag[rank] = ++epoch in every rank's arena (one thread calls this).
SW_DEVICE void ep_signal_all(const unsigned long long* bases, long long flag_off, int world,
                             int rank, uint32_t* epoch) {
  const uint32_t e = *epoch + 1;
  *epoch = e;
  __threadfence_system();
  for (int o = 0; o < world; ++o)
    st_release_sys(reinterpret_cast<uint32_t*>(bases[o] + flag_off) + rank, e);
}

// "Last CTA done" completion signal: every thread of every CTA calls this at
// the very end; the CTA that finishes last raises the flags.  `ctl[0]` is the
// done counter, `ctl[1]` the epoch.  One system-scope fence per CTA, after
// the CTA barrier, publishes all of the CTA's stores (peer stores included)
// before its count: the barrier orders the other threads' stores before
// thread 0's fence, which is cumulative.
SW_DEVICE void ep_grid_done_signal(int* ctl, const unsigned long long* bases, long long flag_off,
                                   int world, int rank) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const int prev = atomicAdd(&ctl[0], 1);
    if (prev == (int)(gridDim.x * gridDim.y * gridDim.z) - 1) {
      ctl[0] = 0;
      ep_signal_all(bases, flag_off, world, rank, reinterpret_cast<uint32_t*>(&ctl[1]));
    }
  }
}

}  // namespace swarm
