// Allocation-free variant of the Q4_K tensor-core GEMM entry point: the
// stream-K partial sums and the status word live in a file-scope device
// array instead of caller-provided or allocated scratch.  See qgemm_noalloc.h
// for who needs this and the rules that come with it.  No counterpart in the
// reference project.
#include "qgemm_noalloc.h"

#include "gemm_out.cuh"
#include "kernels.h"

// Fixed scratch: partial sums followed by the 8-int status word.  Every device
// that loads the library holds it until process exit.
static __device__ __align__(256) unsigned char g_noalloc_scratch[SWARM_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;
// Device address of g_noalloc_scratch per device (the host-side symbol is only
// a stand-in; it must never be passed to a kernel).  These caches are written
// without a lock: two threads setting up the same device at once both store
// the same values, so the race is benign.
void* g_scratch_dev[kMaxDevices] = {nullptr};
int g_num_sms[kMaxDevices] = {0};

int* status_of(int dev) {
  return reinterpret_cast<int*>(static_cast<unsigned char*>(g_scratch_dev[dev]) +
                                SWARM_NOALLOC_SCRATCH_FLOATS * 4u);
}

int setup_device(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return SWARM_NOALLOC_ERR_SETUP;
  if (g_scratch_dev[dev] != nullptr) return SWARM_NOALLOC_OK;
  // Called with `dev` current (the caller's current device).
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr)
    return SWARM_NOALLOC_ERR_SETUP;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
    return SWARM_NOALLOC_ERR_SETUP;
  g_num_sms[dev] = sms;
  g_scratch_dev[dev] = p;
  return SWARM_NOALLOC_OK;
}

}  // namespace

extern "C" long long swarm_q4k_gemm_noalloc_scratch_need(int rows, int K, int T) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return SWARM_NOALLOC_ERR_SETUP;
  if (setup_device(dev) != SWARM_NOALLOC_OK) return SWARM_NOALLOC_ERR_SETUP;
  if (rows <= 0 || K <= 0 || T <= 0 || rows % 128 || K % 256) return SWARM_NOALLOC_ERR_SHAPE;
  int N, ntt, kb, upc, ctas;
  long total;
  size_t need;
  q4k_tc_plan(rows, K, T, g_num_sms[dev], &N, &ntt, &kb, &total, &upc, &ctas, &need);
  return (long long)need * 4;
}

extern "C" int swarm_q4k_gemm_noalloc(const void* w_packed, int rows, int K, const __half* x,
                                      int x_stride, int T, float* out, int out_stride,
                                      cudaStream_t stream) {
  if (rows <= 0 || K <= 0 || T <= 0 || rows % 128 || K % 256) return SWARM_NOALLOC_ERR_SHAPE;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return SWARM_NOALLOC_ERR_SETUP;
  const int rc_setup = setup_device(dev);
  if (rc_setup != SWARM_NOALLOC_OK) return rc_setup;
  int N, ntt, kb, upc, ctas;
  long total;
  size_t need;
  q4k_tc_plan(rows, K, T, g_num_sms[dev], &N, &ntt, &kb, &total, &upc, &ctas, &need);
  if (need > SWARM_NOALLOC_SCRATCH_FLOATS) return SWARM_NOALLOC_ERR_TOO_LARGE;

  float* partials = static_cast<float*>(g_scratch_dev[dev]);
  int* status = status_of(dev);
  // The status word must start at zero for every call (timed-out waits set it).
  if (cudaMemsetAsync(status, 0, 32, stream) != cudaSuccess) return SWARM_NOALLOC_ERR_LAUNCH;
  swarm::GemmOut g{};
  int rc = launch_qgemm_q4k_tc(w_packed, rows, K, x, x_stride, T, partials,
                               SWARM_NOALLOC_SCRATCH_FLOATS, g_num_sms[dev], status, &g, stream);
  if (rc != 0) return SWARM_NOALLOC_ERR_LAUNCH;
  launch_epi_copy(g, nullptr, out, out_stride, stream);
  return cudaPeekAtLastError() == cudaSuccess ? SWARM_NOALLOC_OK : SWARM_NOALLOC_ERR_LAUNCH;
}

extern "C" int swarm_q4k_gemm_noalloc_status(int* host_status8, cudaStream_t stream) {
  if (host_status8 == nullptr) return SWARM_NOALLOC_ERR_SHAPE;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return SWARM_NOALLOC_ERR_SETUP;
  const int rc_setup = setup_device(dev);
  if (rc_setup != SWARM_NOALLOC_OK) return rc_setup;
  // Ordered after the caller's GEMM on `stream`; the host buffer is pageable
  // memory of the caller's, so the copy is synchronous with respect to it.
  if (cudaMemcpyAsync(host_status8, status_of(dev), 32, cudaMemcpyDeviceToHost, stream) !=
          cudaSuccess ||
      cudaStreamSynchronize(stream) != cudaSuccess)
    return SWARM_NOALLOC_ERR_LAUNCH;
  return host_status8[0] == 0 ? SWARM_NOALLOC_OK : SWARM_NOALLOC_ERR_KERNEL;
}

extern "C" const char* swarm_q4k_gemm_noalloc_error(int code) {
  switch (code) {
    case SWARM_NOALLOC_OK: return "ok";
    case SWARM_NOALLOC_ERR_TOO_LARGE:
      return "problem too large: its stream-K partial sums exceed the 16 MiB static scratch "
             "(see swarm_q4k_gemm_noalloc_scratch_need); use the regular entry point with a "
             "caller-provided workspace";
    case SWARM_NOALLOC_ERR_SHAPE: return "bad shape: need rows % 128 == 0, K % 256 == 0, T > 0";
    case SWARM_NOALLOC_ERR_SETUP:
      return "setup failed: could not get the device address of the static scratch or the SM count";
    case SWARM_NOALLOC_ERR_LAUNCH: return "kernel launch failed";
    case SWARM_NOALLOC_ERR_KERNEL:
      return "the GEMM gave up on a bounded wait inside the kernel; the output of that call is "
             "invalid (status word: [0] code, [1] block, [2..3] details)";
    default: return "unknown error code";
  }
}
