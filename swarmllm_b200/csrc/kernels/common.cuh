// Shared device helpers for the sm_100a kernels of swarmllm_b200.
//
// Every kernel in this directory is plain CUDA C++ with no torch headers; the
// launchers take raw device pointers plus a cudaStream_t and are bound to
// PyTorch in csrc/bindings/torch_ops.cpp.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#define SW_DEVICE __device__ __forceinline__
#define SW_HOST_DEVICE __host__ __device__ __forceinline__

namespace swarm {

constexpr int kWarp = 32;

// Programmatic dependent launch (PDL).  The decode-path kernels are launched
// with programmatic stream serialisation: they may start while the kernel
// before them is still running.  Every kernel calls pdl_trigger() first thing,
// which lets the next grid launch as soon as every CTA of the current one is
// running, and pdl_wait() before it reads anything an earlier kernel wrote
// (it returns once the previous grid -- and through it every earlier one --
// has completed and its writes are visible).  The weight-streaming GEMMs
// stream their first weight tiles before waiting; the epilogue-type kernels
// wait at once, so they only hide their launch latency.  Both calls are
// no-ops for launches without the attribute.
SW_DEVICE void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
SW_DEVICE void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Host: whether launches opt into PDL (SWARMLLM_PDL=0 turns it off).
bool pdl_enabled();

// Launch `kernel` with programmatic stream serialisation (when enabled).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

// The same with a thread-block cluster of `cluster_x` CTAs (1: none).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block,
                                      size_t smem, cudaStream_t s, int cluster_x,
                                      Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

// cudaFuncSetAttribute applies to the device current at the call, so a launcher
// that raises a kernel's dynamic shared-memory limit must do it once on every
// device it launches on.  `done` is the launcher's bit mask of devices already
// set (up to 64 devices); returns false if the attribute could not be set.
template <typename Kernel>
inline bool smem_attr_once(Kernel* fn, int bytes, unsigned long long* done) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  const unsigned long long bit = 1ull << dev;
  if (__atomic_load_n(done, __ATOMIC_ACQUIRE) & bit) return true;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
    return false;
  __atomic_fetch_or(done, bit, __ATOMIC_RELEASE);
  return true;
}

SW_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

SW_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum; `smem` must hold >= 32 floats.  All threads get the result.
SW_DEVICE float block_sum(float v, float* smem) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) smem[wid] = v;
  __syncthreads();
  float r = (threadIdx.x < nw) ? smem[threadIdx.x] : 0.f;
  if (wid == 0) {
    r = warp_sum(r);
    if (lane == 0) smem[0] = r;
  }
  __syncthreads();
  return smem[0];
}

SW_DEVICE float block_max(float v, float* smem) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) smem[wid] = v;
  __syncthreads();
  float r = (threadIdx.x < nw) ? smem[threadIdx.x] : -INFINITY;
  if (wid == 0) {
    r = warp_max(r);
    if (lane == 0) smem[0] = r;
  }
  __syncthreads();
  return smem[0];
}

SW_DEVICE float to_f(float x) { return x; }
SW_DEVICE float to_f(__half x) { return __half2float(x); }
SW_DEVICE float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T> SW_DEVICE T from_f(float x);
template <> SW_DEVICE float from_f<float>(float x) { return x; }
template <> SW_DEVICE __half from_f<__half>(float x) { return __float2half_rn(x); }
template <> SW_DEVICE __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// Half stored as raw uint16 bits (GGUF block scales).
SW_DEVICE float half_bits_to_f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

SW_DEVICE float silu(float x) { return x / (1.f + __expf(-x)); }

}  // namespace swarm

// Host-side launch check: records the last launch error without syncing.
#define SW_LAUNCH_CHECK() do { (void)cudaPeekAtLastError(); } while (0)
