// Expert-parallel all-to-all for the MoE layers, over NVLink peer memory.
//
// Every rank owns E_loc = E / W consecutive experts and one "arena" of device
// memory that all ranks map (CUDA IPC).  Arena layout (same offsets on every
// rank, in bytes):
//   recv_x   [W][cap][H]  16-bit   token rows sent to this rank's experts
//   recv_ret [W][cap]     int32    return address of each row: src << 24 | slot
//   recv_cnt [W][E_loc]   int32    per-source token counts per local expert
//   comb     [cap][H]     fp32     expert outputs of this rank's own (token, k) slots
//   flags_d  [W]          uint32   dispatch done, one word per source
//   flags_c  [W]          uint32   combine done, one word per owner
// cap = max (token, k) pairs one rank sends in a layer.
//
// Per MoE layer (all kernels on the compute stream, graph-capturable):
//   source:  ep_send_counts  per-owner exclusive scan of the local expert
//                            counts (sets the dispatch cursors) and P2P store
//                            of the counts into every owner's recv_cnt
//            ep_dispatch     one warp per (token, k) pair: reserve a row in
//                            the owner's region, P2P store of the row and its
//                            return address; the last CTA to finish raises
//                            flags_d[rank] on every owner
//   owner:   ep_wait         bounded wait for all W dispatch flags
//            ep_plan_owner   tile list over (local expert, source) segments
//            moe_gemm_tc     gate|up (SwiGLU) then down, whose epilogue stores
//                            each result row straight into the source's comb
//                            (P2P) and whose last CTA raises flags_c[rank] on
//                            every source
//   source:  ep_wait         bounded wait for all W combine flags
//            moe_combine     weighted sum of the k rows per token (local)
// Flags carry an epoch that both sides count in lockstep, so nothing is reset
// between layers.  Every wait gives up after a deadline and records an error
// in the status word instead of spinning forever.
//
// No TMA (and no multicast) touches peer memory: peers are only written with
// plain stores, and the grouped GEMM reads its own arena through TMA.
// Reference: the reference keeps every expert of a layer on the node holding
// the layer (no expert parallelism; src/inference/layers/moe.rs);
// the closest behaviour is its network TP all-reduce (src/network/tp_*.rs).
#include "kernels.h"
#include "common.cuh"
#include "tc_utils.cuh"
#include "ep_common.cuh"

namespace swarm {

struct EpLayout {
  long long recv_x, recv_ret, recv_cnt, comb, flags_d, flags_c, total;
};

// local control words (int32[16] on the device, zero-initialised)
//   [0] dispatch done counter  [1] dispatch signal epoch  [2] dispatch wait epoch
//   [3] combine done counter   [4] combine signal epoch   [5] combine wait epoch

// One CTA, E threads (E <= 1024).
__global__ void ep_send_counts_kernel(int* __restrict__ counts, int E, int e_loc, EpPeers peers,
                                      EpLayout lay, int world, int rank,
                                      int* __restrict__ cursor) {
  const int e = threadIdx.x;  // launched with exactly E threads
  const int o = e / e_loc, el = e - o * e_loc;
  int off = 0;
  for (int j = o * e_loc; j < e; ++j) off += counts[j];  // E_loc <= 128: short
  const int c = counts[e];
  __syncthreads();  // every count is read before any is cleared
  int* rc = reinterpret_cast<int*>(peers.base[o] + lay.recv_cnt);
  rc[rank * e_loc + el] = c;
  cursor[e] = off;
  counts[e] = 0;
}

template <typename XT>
__global__ void ep_dispatch_kernel(const __half* __restrict__ x, int x_stride, int H,
                                   const int32_t* __restrict__ ids, int P, int k, int e_loc,
                                   int cap, int* __restrict__ cursor, EpPeers peers, EpLayout lay,
                                   int world, int rank, int* __restrict__ ctl) {
  const int p = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (p < P) {
    const int e = ids[p];
    const int o = e / e_loc;
    int pos = 0;
    if (lane == 0) pos = atomicAdd(&cursor[e], 1);
    pos = __shfl_sync(0xffffffffu, pos, 0);
    const size_t row = (size_t)rank * cap + pos;
    XT* dst = reinterpret_cast<XT*>(peers.base[o] + lay.recv_x) + row * H;
    const __half* src = x + (size_t)(p / k) * x_stride;
    for (int i = lane * 2; i < H; i += 64) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(src + i));
      dst[i] = from_f<XT>(f.x);
      dst[i + 1] = from_f<XT>(f.y);
    }
    if (lane == 0) reinterpret_cast<int*>(peers.base[o] + lay.recv_ret)[row] = (rank << 24) | p;
  }
  ep_grid_done_signal(ctl, peers.base, lay.flags_d, world, rank);
}

// One CTA, `world` threads: wait until flags[src] reaches this side's next epoch.
__global__ void ep_wait_kernel(const uint32_t* flags, int world, int* __restrict__ ctl,
                               int wait_slot, int* __restrict__ status, int code,
                               unsigned long long timeout_ns) {
  __shared__ int ok_all;
  const uint32_t want = (uint32_t)ctl[wait_slot] + 1;
  if (threadIdx.x == 0) ok_all = 1;
  __syncthreads();
  if (threadIdx.x < world) {
    const unsigned long long t0 = tc::globaltimer();
    bool ok = true;
    int n = 0;
    while ((int)(ld_acquire_sys(flags + threadIdx.x) - want) < 0) {
      if ((++n & 63) == 0 && tc::globaltimer() - t0 > timeout_ns) {
        ok = false;
        break;
      }
    }
    if (!ok) {
      ok_all = 0;
      if (status && atomicCAS(&status[0], 0, code) == 0) {
        status[1] = -1;
        status[2] = threadIdx.x;
        status[3] = (int)want;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) ctl[wait_slot] = (int)want;
}

// One CTA (world * e_loc <= 1024 threads): tiles over (local expert, source)
// segments, expert-major so that tiles of one expert are adjacent.
__global__ void ep_plan_owner_kernel(const int* __restrict__ recv_cnt, int world, int e_loc,
                                     int cap, int N, int4* __restrict__ tiles,
                                     int* __restrict__ n_tiles, int max_tiles,
                                     int* __restrict__ status) {
  __shared__ int s_t[32];
  const int seg = threadIdx.x;  // = el * world + src
  const int nseg = world * e_loc;
  const int lane = seg & 31, warp = seg >> 5;
  int c = 0, off = 0, el = 0, src = 0;
  if (seg < nseg) {
    el = seg / world;
    src = seg - el * world;
    c = recv_cnt[src * e_loc + el];
    for (int j = 0; j < el; ++j) off += recv_cnt[src * e_loc + j];
  }
  const int nt = (c + N - 1) / N;
  int it = nt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int b = __shfl_up_sync(0xffffffffu, it, o);
    if (lane >= o) it += b;
  }
  if (lane == 31) s_t[warp] = it;
  __syncthreads();
  if (warp == 0) {
    int b = lane < (int)((blockDim.x + 31) >> 5) ? s_t[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, b, o);
      if (lane >= o) b += y;
    }
    s_t[lane] = b;
  }
  __syncthreads();
  const int base_t = (warp ? s_t[warp - 1] : 0) + it - nt;
  for (int j = 0; j < nt; ++j)
    if (base_t + j < max_tiles)
      tiles[base_t + j] = make_int4(el, src * cap + off + j * N, min(N, c - j * N), 0);
  if (seg == (int)blockDim.x - 1) {
    const int total = s_t[((blockDim.x + 31) >> 5) - 1];
    *n_tiles = min(total, max_tiles);
    if (total > max_tiles && status) status[6] = total;
  }
}

}  // namespace swarm

using namespace swarm;

// ---------------------------------------------------------------- host side
static EpLayout ep_layout(int world, int cap, int H, int e_loc) {
  EpLayout l{};
  long long o = 0;
  auto take = [&](long long bytes) {
    const long long at = o;
    o += (bytes + 255) / 256 * 256;
    return at;
  };
  l.recv_x = take((long long)world * cap * H * 2);
  l.recv_ret = take((long long)world * cap * 4);
  l.recv_cnt = take((long long)world * e_loc * 4);
  l.comb = take((long long)cap * H * 4);
  l.flags_d = take((long long)world * 4);
  l.flags_c = take((long long)world * 4);
  l.total = o;
  return l;
}

long long ep_arena_bytes(int world, int cap, int H, int e_loc) {
  return ep_layout(world, cap, H, e_loc).total;
}

void ep_arena_offsets(int world, int cap, int H, int e_loc, long long* out6) {
  const EpLayout l = ep_layout(world, cap, H, e_loc);
  out6[0] = l.recv_x;
  out6[1] = l.recv_ret;
  out6[2] = l.recv_cnt;
  out6[3] = l.comb;
  out6[4] = l.flags_d;
  out6[5] = l.flags_c;
}

int ep_arena_alloc(long long bytes, void** ptr, void* handle64) {
  if (cudaMalloc(ptr, (size_t)bytes) != cudaSuccess) return -1;
  if (cudaMemset(*ptr, 0, (size_t)bytes) != cudaSuccess) return -2;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, *ptr) != cudaSuccess) return -3;
  memcpy(handle64, &h, sizeof(h));
  return 0;
}

int ep_arena_open(const void* handle64, void** ptr) {
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof(h));
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? 0 : -1;
}

int ep_arena_close(void* ptr, int own) {
  if (own) return cudaFree(ptr) == cudaSuccess ? 0 : -1;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? 0 : -1;
}

static EpPeers make_peers(const unsigned long long* bases, int world) {
  EpPeers p{};
  for (int i = 0; i < world && i < 8; ++i) p.base[i] = bases[i];
  return p;
}

int launch_ep_dispatch(const __half* x, int x_stride, int H, const int32_t* ids, int P, int k,
                       int* counts, int E, int e_loc, int cap, int* cursor,
                       const unsigned long long* bases, int world, int rank, int x_bf16,
                       int* ctl, cudaStream_t s) {
  if (world > 8 || E > 1024 || e_loc * world != E) return -1;
  if (P > cap || H % 2) return -2;
  const EpLayout lay = ep_layout(world, cap, H, e_loc);
  const EpPeers peers = make_peers(bases, world);
  ep_send_counts_kernel<<<1, E, 0, s>>>(counts, E, e_loc, peers, lay, world, rank, cursor);
  const int warps = 8;
  const unsigned grid = (unsigned)((P + warps - 1) / warps > 0 ? (P + warps - 1) / warps : 1);
  if (x_bf16)
    ep_dispatch_kernel<__nv_bfloat16><<<grid, 32 * warps, 0, s>>>(
        x, x_stride, H, ids, P, k, e_loc, cap, cursor, peers, lay, world, rank, ctl);
  else
    ep_dispatch_kernel<__half><<<grid, 32 * warps, 0, s>>>(x, x_stride, H, ids, P, k, e_loc, cap,
                                                           cursor, peers, lay, world, rank, ctl);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -3;
}

int launch_ep_wait(unsigned long long own_base, int world, int cap, int H, int e_loc, int which,
                   int* ctl, int* status, cudaStream_t s, long long timeout_ns) {
  const EpLayout lay = ep_layout(world, cap, H, e_loc);
  const uint32_t* flags =
      reinterpret_cast<const uint32_t*>(own_base + (which == 0 ? lay.flags_d : lay.flags_c));
  ep_wait_kernel<<<1, 32, 0, s>>>(flags, world, ctl, which == 0 ? 2 : 5, status,
                                  which == 0 ? 61 : 62,
                                  timeout_ns > 0 ? (unsigned long long)timeout_ns
                                                 : tc::kWaitTimeoutNs);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -1;
}

int launch_ep_plan_owner(unsigned long long own_base, int world, int cap, int H, int e_loc,
                         int tok_tile, void* tiles, int* n_tiles, int max_tiles, int* status,
                         cudaStream_t s) {
  const int nseg = world * e_loc;
  if (nseg > 1024) return -1;
  const EpLayout lay = ep_layout(world, cap, H, e_loc);
  const int threads = (nseg + 31) / 32 * 32;
  ep_plan_owner_kernel<<<1, threads, 0, s>>>(
      reinterpret_cast<const int*>(own_base + lay.recv_cnt), world, e_loc, cap, tok_tile,
      (int4*)tiles, n_tiles, max_tiles, status);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -2;
}

int launch_flag_wait(const void* flags, int world, int* ctl, int slot, int* status, int code,
                     cudaStream_t s, long long timeout_ns) {
  if (world < 1 || world > 32) return -1;
  ep_wait_kernel<<<1, 32, 0, s>>>(reinterpret_cast<const uint32_t*>(flags), world, ctl, slot,
                                  status, code,
                                  timeout_ns > 0 ? (unsigned long long)timeout_ns
                                                 : tc::kWaitTimeoutNs);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -2;
}
