// LoRA adapters applied per row: delta[t] = scale[a] * B[a] (A[a] x[t]) for the
// adapter a = ids[t] of token row t (no delta for ids[t] < 0), so requests
// with different adapters (or none) share one batch.  The dense delta is
// added to the base GEMM's result by every epilogue that reads it (GemmOut.add).
//
//   lora_shrink  one warp per (row, rank index): u[t][j] = A[a][j] . x[t]
//   lora_expand  one thread per (row, output): delta = scale * B[a][i] . u[t]
//
// A [M][R][K] fp16, B [M][rows][R] fp16 (M adapters stacked, R = padded rank).
// Reference: per-request LoRA adapters from GGUF (src/inference/lora.rs).
#include "kernels.h"
#include "common.cuh"

namespace swarm {

__global__ void lora_shrink_kernel(const __half* __restrict__ x, int x_stride, int K,
                                   const int32_t* __restrict__ ids, const __half* __restrict__ A,
                                   int R, int T, float* __restrict__ u) {
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= T * R) return;
  const int t = w / R, j = w - t * R;
  const int a = ids[t];
  float acc = 0.f;
  if (a >= 0) {
    const __half* ar = A + ((size_t)a * R + j) * K;
    const __half* xr = x + (size_t)t * x_stride;
    for (int k = lane * 2; k < K; k += 64) {
      const float2 av = __half22float2(*reinterpret_cast<const __half2*>(ar + k));
      const float2 xv = __half22float2(*reinterpret_cast<const __half2*>(xr + k));
      acc += av.x * xv.x + av.y * xv.y;
    }
    acc = warp_sum(acc);
  }
  if (lane == 0) u[(size_t)t * R + j] = acc;
}

__global__ void lora_expand_kernel(const float* __restrict__ u, const int32_t* __restrict__ ids,
                                   const __half* __restrict__ B, const float* __restrict__ scale,
                                   int R, int rows, int T, float* __restrict__ delta) {
  const int t = blockIdx.y;
  const int a = ids[t];
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < rows; i += gridDim.x * blockDim.x) {
    float acc = 0.f;
    if (a >= 0) {
      const __half* br = B + ((size_t)a * rows + i) * R;
      for (int j = 0; j < R; ++j) acc += __half2float(br[j]) * u[(size_t)t * R + j];
      acc *= scale[a];
    }
    delta[(size_t)t * rows + i] = acc;
  }
}

}  // namespace swarm

using namespace swarm;

int launch_lora(const __half* x, int x_stride, int K, const int32_t* ids, int T, const __half* A,
                const __half* B, const float* scale, int R, int rows, float* u, float* delta,
                cudaStream_t s) {
  if (T <= 0) return 0;
  if (K % 2) return -1;
  const int warps = T * R;
  lora_shrink_kernel<<<(warps + 7) / 8, 256, 0, s>>>(x, x_stride, K, ids, A, R, T, u);
  dim3 g((rows + 255) / 256 < 64 ? (rows + 255) / 256 : 64, T);
  lora_expand_kernel<<<g, 256, 0, s>>>(u, ids, B, scale, R, rows, T, delta);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -2;
}
