// Quantized matmul on the host CPU over GGUF blocks (Q4_K, Q6_K, Q8_0, Q4_0,
// IQ4_NL, IQ4_XS, MXFP4).
#pragma once
#include <cstdint>

namespace swarm_native {

// ggml type ids of the formats the CPU kernel reads
constexpr int kGgmlQ4_0 = 2;
constexpr int kGgmlQ8_0 = 8;
constexpr int kGgmlQ4_K = 12;
constexpr int kGgmlQ6_K = 14;
constexpr int kGgmlIQ4_NL = 20;
constexpr int kGgmlIQ4_XS = 23;
constexpr int kGgmlMXFP4 = 39;

// out [T, rows] = x [T, K] . W^T, W = `rows` rows of GGUF blocks of `type`.
// Returns 0, or < 0 for an unsupported type or K.
int cpu_qmatmul(const uint8_t* w, int type, int rows, int K, const float* x, int T, float* out);

// out [rows, K] fp32 = the weight's values (the blocks' scales applied).
int cpu_dequant(const uint8_t* w, int type, int rows, int K, float* out);

// "avx512vnni" or "generic": the path cpu_qmatmul takes on this CPU
// (SWARMLLM_CPU_ISA=generic forces the portable one).
const char* cpu_qmatmul_isa();

}  // namespace swarm_native
