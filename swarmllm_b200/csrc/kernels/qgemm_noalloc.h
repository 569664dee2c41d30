// Allocation-free entry point for the Q4_K tensor-core GEMM.
//
// This entry point has no counterpart in the reference project; it exists for
// callers of this library that are not allowed to allocate device memory,
// for example code running inside a host framework that owns every device
// allocation (a custom allocator or memory pool it does not let plug-ins call
// into), plug-ins that may only use the buffers they are handed, or code
// paths that must never trigger an implicit device-wide synchronisation
// through cudaMalloc/cudaFree.
//
// It computes  out[t][r] = sum_k W[r][k] * x[t][k]  exactly like the regular
// path (launch_qgemm_q4k_tc followed by the logits-copy epilogue), but its
// scratch -- the stream-K partial sums and the kernel's status word -- lives
// in a fixed file-scope device array of SWARM_NOALLOC_SCRATCH_BYTES (16 MiB
// plus 32 bytes), which every GPU that loads this library keeps until the
// process exits.  Nothing is allocated: no cudaMalloc, no cudaFree, no
// allocating library routine.
//
// Rules for callers:
//  * Inputs and outputs are the caller's device buffers: w_packed is a Q4_K
//    weight already repacked for the tensor-core GEMM (launch_q4k_repack),
//    x is fp16 [T, K] (row stride x_stride elements), out is fp32 [T, rows]
//    (row stride out_stride elements).  rows % 128 == 0, K % 256 == 0.
//  * The first call on a device finds the device address of the scratch array
//    (cudaGetSymbolAddress, with that device current) and caches it.  Make
//    that first call on each device before any stream capture begins.
//  * All calls on a device share the one scratch array.  Two calls whose work
//    overlaps on the GPU (e.g. on different streams without ordering between
//    them) race on it; serialise such calls.  The status word is cleared at
//    the start of every call; the partial sums are always written before they
//    are read, so nothing else needs clearing.
//  * A problem whose partial sums need more than the scratch holds is
//    rejected with SWARM_NOALLOC_ERR_TOO_LARGE before anything is launched.
//  * swarm_q4k_gemm_noalloc returns once the work is queued; it cannot see
//    what happens on the GPU.  Every wait inside the GEMM is bounded, and a
//    wait that runs out records a code in the status word and ends the kernel
//    early.  swarm_q4k_gemm_noalloc_status(host_status8, stream) waits for the
//    stream, copies that status word (8 ints) to the caller's host buffer and
//    returns SWARM_NOALLOC_ERR_KERNEL when it is set: the output of that call
//    is then invalid.  Read it before the next call on the device, which
//    clears the word again.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>

#define SWARM_NOALLOC_SCRATCH_FLOATS (4u * 1024u * 1024u)  // 16 MiB of partial sums
#define SWARM_NOALLOC_SCRATCH_BYTES (SWARM_NOALLOC_SCRATCH_FLOATS * 4u + 32u)

#define SWARM_NOALLOC_OK 0
#define SWARM_NOALLOC_ERR_TOO_LARGE -10   // partial sums exceed the scratch array
#define SWARM_NOALLOC_ERR_SHAPE -11       // rows % 128 or K % 256 not zero, or T <= 0
#define SWARM_NOALLOC_ERR_SETUP -12       // cudaGetSymbolAddress / device query failed
#define SWARM_NOALLOC_ERR_LAUNCH -13      // the GEMM or epilogue launch failed
#define SWARM_NOALLOC_ERR_KERNEL -14      // the last call's kernel recorded an error (status)

#ifdef __cplusplus
extern "C" {
#endif

__attribute__((visibility("default"))) int swarm_q4k_gemm_noalloc(
    const void* w_packed, int rows, int K, const __half* x, int x_stride, int T, float* out,
    int out_stride, cudaStream_t stream);

// Status of the most recent call on the current device: waits for `stream`,
// copies the 8-int status word into host_status8 and returns SWARM_NOALLOC_OK
// (status clear: the output is valid) or SWARM_NOALLOC_ERR_KERNEL (invalid).
__attribute__((visibility("default"))) int swarm_q4k_gemm_noalloc_status(int* host_status8,
                                                                         cudaStream_t stream);

// Human-readable text for a return code of swarm_q4k_gemm_noalloc.
__attribute__((visibility("default"))) const char* swarm_q4k_gemm_noalloc_error(int code);

// Bytes of partial-sum scratch a (rows, K, T) problem needs on this device
// (compare with SWARM_NOALLOC_SCRATCH_FLOATS * 4); negative on error.
__attribute__((visibility("default"))) long long swarm_q4k_gemm_noalloc_scratch_need(int rows,
                                                                                     int K, int T);

#ifdef __cplusplus
}
#endif
