// Shared helpers of the torch bindings (module swarmllm_b200._C).
#pragma once
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <execinfo.h>
#include <signal.h>
#include <unistd.h>

#include <cstdlib>

#include "kernels.h"
#include "gemm_out.cuh"

namespace py = pybind11;
using at::Tensor;
using OptT = std::optional<Tensor>;

#define CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define CHECK_CONTIG(x) TORCH_CHECK((x).is_contiguous(), #x " must be contiguous")
#define CHECK_DT(x, dt) TORCH_CHECK((x).scalar_type() == (dt), #x " has wrong dtype")

static inline cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

template <typename T>
static inline T* ptr_or_null(const OptT& t) {
  return (t.has_value() && t->defined()) ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}

// A GEMM result: the fp32 workspace plus how to read it (see gemm_out.cuh).
struct GemmResult {
  swarm::GemmOut g{};
  Tensor ws;  // keeps the buffer alive
};

static inline int num_sms_of(const Tensor& t) {
  static int cached[64] = {0};
  int dev = t.get_device();
  if (dev < 0 || dev >= 64) dev = 0;
  if (!cached[dev]) {
    cudaDeviceProp p;
    cudaGetDeviceProperties(&p, dev);
    cached[dev] = p.multiProcessorCount;
  }
  return cached[dev];
}

