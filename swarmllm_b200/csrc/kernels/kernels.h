// Host-side launchers of the sm_100a kernels.  Plain pointers + stream; no
// torch types, so the kernels build without torch headers and the same entry
// points can be called from C/C++ hosts.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stddef.h>
#include <stdint.h>

namespace swarm {
struct GemmOut;
}

// ---- elementwise / epilogues (elementwise.cu) ------------------------------
void launch_embed_gather(const void* table, int type, int hidden, const int32_t* ids, int n,
                         float* out, cudaStream_t s);
void launch_rmsnorm(const float* x, const float* w, __half* out, int rows, int dim, float eps,
                    cudaStream_t s);
void launch_epi_residual_rmsnorm(const swarm::GemmOut& g, float* residual, const float* bias,
                                 const float* w, __half* out, float eps, int out_stride,
                                 cudaStream_t s, const float* post_w = nullptr);
void launch_epi_rope_kv(const swarm::GemmOut& g, const float* bias, const int32_t* positions,
                        const int32_t* slots, const float* inv_freq, int n_q, int n_kv,
                        int head_dim, int rope_dim, int neox, float attn_factor, __half* q_out,
                        __half* k_cache, __half* v_cache, int page_size, const float* q_norm_w,
                        const float* k_norm_w, float norm_eps, __half* gate_out, cudaStream_t s);
void launch_epi_swiglu(const swarm::GemmOut& g, const float* bias, int F, int kind,
                       int interleaved, float alpha, float limit, __half* out, cudaStream_t s);
void launch_epi_copy(const swarm::GemmOut& g, const float* bias, float* out, int out_stride,
                     cudaStream_t s);
void launch_f32_to_f16(const float* x, __half* y, size_t n, cudaStream_t s);

// ---- quantized GEMM ---------------------------------------------------------
int launch_qmatmul_simt(const void* w, int type, int rows, int K, const __half* x, int x_stride,
                        int T, float* out, int out_stride, cudaStream_t s);
int q4k_tc_tok_tile(int T);
// Weight formats of the repacked quantized GEMM (qfmt.cuh): the GGML type
// number maps to fmt 0 = Q4_K, 1 = Q6_K, 2 = Q8_0; -1 = no tensor-core path.
constexpr int qfmt_of_ggml(int ggml_type) {
  return ggml_type == 12 ? 0 : (ggml_type == 14 ? 1 : (ggml_type == 8 ? 2 : -1));
}
constexpr int qfmt_row_bytes(int fmt) { return fmt == 0 ? 144 : (fmt == 1 ? 224 : 272); }
// Decode at <= kQGemvMaxT tokens runs the CUDA-core GEMV (qgemv_q4k.cu) with
// qgemv_ctas_per_sm(fmt, T) CTAs per SM; the plan below accounts for it.
constexpr int kQGemvMaxT = 2;
constexpr int qgemv_ctas_per_sm(int fmt, int T) {
  return fmt == 0 ? (T == 1 ? 5 : 4) : (fmt == 1 ? 3 : (T == 1 ? 3 : 2));
}
constexpr int q4k_gemv_ctas_per_sm(int T) { return qgemv_ctas_per_sm(0, T); }
int q4k_gemv_max_t();          // kQGemvMaxT unless SWARMLLM_QGEMV_MAX_T overrides (0 = off)
int q4k_plan_max_ctas(int T, int num_sms, int fmt = 0);
int q4k_gemv_occupancy(int T, int fmt = 0);  // resident GEMV CTAs per SM (diagnostics)
int launch_qgemv_q4k(const void* w_packed, int rows, int K, const __half* x, int x_stride, int T,
                     float* ws, int ksb, long total_units, int upc, int ctas, int* status,
                     const unsigned long long* peer_ws, int n_peers, int* sig_ctl,
                     const unsigned long long* sig_bases, long long sig_flag_off, int sig_rank,
                     cudaStream_t s, int owner_tiles = 0, int fmt = 0,
                     const void* w_b = nullptr, int fmt_b = -1, int split_tile = 0);
void q4k_tc_plan(int rows, int K, int T, int num_sms, int* tok_tile, int* n_tok_tiles, int* ksb,
                 long* total_units, int* upc, int* n_ctas, size_t* ws_floats, int fmt = 0);
// fmt selects the repacked weight format (qfmt_of_ggml); the name keeps the
// format the kernel started with.  Mixed-format GEMM (a Q4_K_M checkpoint's
// q|k|v, whose v rows are Q6_K): row tiles [0, split_tile) come from w_packed
// in fmt, the rest from w_b in fmt_b (only fmt Q4_K + fmt_b Q6_K is built).
int launch_qgemm_q4k_tc(const void* w_packed, int rows, int K, const __half* x, int x_stride,
                        int T, float* ws, size_t ws_floats_avail, int num_sms, int* status,
                        swarm::GemmOut* out, cudaStream_t s,
                        const unsigned long long* peer_ws = nullptr, int n_peers = 0,
                        int* sig_ctl = nullptr, const unsigned long long* sig_bases = nullptr,
                        long long sig_flag_off = 0, int sig_rank = 0, int owner_tiles = 0,
                        int fmt = 0, const void* w_b = nullptr, int fmt_b = -1,
                        int split_tile = 0);
void qgemm_set_trace(void* buf);
// Dense fp16 weights on tcgen05 (dense_gemm_tc.cu); same workspace contract.
void dense_tc_plan(int rows, int K, int T, int num_sms, int* tok_tile, int* n_tok_tiles, int* kb,
                   long* total_units, int* upc, int* n_ctas, size_t* ws_floats);
int launch_dense_gemm_tc(const __half* w, int rows, int K, int w_stride, const __half* x,
                         int x_stride, int T, float* ws, size_t ws_floats_avail, int num_sms,
                         int* status, swarm::GemmOut* out, cudaStream_t s);
int launch_q4k_repack(const void* src, int rows, int K, void* dst, cudaStream_t s);
// GGUF Q6_K / Q8_0 rows -> the tiled layouts of qfmt.cuh (fmt 1 / 2).
int launch_qfmt_repack(int fmt, const void* src, int rows, int K, void* dst, cudaStream_t s);
int make_tmap_2d_16bit(CUtensorMap* map, const void* base, int rows, int cols, int row_stride,
                       int box_rows, int box_cols, int swizzle_bytes);

// ---- attention --------------------------------------------------------------
int launch_decode_attn_simt(const __half* q, const __half* k_cache, const __half* v_cache,
                            const int32_t* block_table, int bt_stride, const int32_t* seq_lens,
                            const uint64_t* tree_mask, const int32_t* tree_start,
                            const float* sinks, int T, int n_q, int n_kv, int head_dim,
                            int page_size, int window, float scale, float softcap,
                            int keys_per_split, int n_splits, float* part_o, float* part_ml,
                            __half* out, cudaStream_t s);

void attn_set_trace(void* buf);
void launch_attn_combine(const float* part_o, const float* part_ml, int rows, int n_splits, int D,
                         const float* sinks, int n_q, __half* out, cudaStream_t s);
int launch_attn_tc(const __half* q, int T, int n_q, const __half* k_cache, const __half* v_cache,
                   long num_pages, int n_kv, int D, const int32_t* group_row0,
                   const int32_t* group_npos, int G, int pos_per_group, const int32_t* block_table,
                   int bt_stride, const int32_t* seq_lens, const uint64_t* tree_mask,
                   const int32_t* tree_start, const float* sinks, int window, float scale,
                   int keys_per_split, int n_splits, __half* out, float* part_o, float* part_ml,
                   int* status, cudaStream_t s);

// ---- sampling -----------------------------------------------------------------
void launch_argmax(const float* logits, int rows, int V, int stride, int32_t* out, float* out_val,
                   cudaStream_t s);
void launch_sample(const float* logits, int rows, int V, int stride, const float* temperature,
                   const int32_t* top_k, const float* top_p, const uint64_t* seeds,
                   const int32_t* positions, int32_t* out, cudaStream_t s);
void launch_philox_uniform(uint64_t seed, const int32_t* positions, int n_pos, int V, float* out,
                           cudaStream_t s);
void launch_apply_penalties(float* logits, int rows, int V, int stride, const int32_t* off,
                            const int32_t* tok, const float* val, cudaStream_t s);

// ---- mixture of experts (moe_tc.cu) -----------------------------------------
// fmt: 0 = Q4_K experts (fp16 activations), 1 = MXFP4 experts (bf16 activations)
// epi: 0 = SwiGLU (gate/up rows interleaved in groups of 16) -> 16-bit H
//      1 = store fp32 rows to out_ptrs[ret >> 24][ret & 0xFFFFFF]
int moe_tok_tile(int pairs, int n_experts);
int moe_max_tiles(int pairs, int n_experts, int tok_tile);
long long moe_packed_bytes(int fmt, int rows, int K);
int launch_mxfp4_repack(const void* src, int rows, int K, void* dst, cudaStream_t s);
// mode 0 softmax over all, 1 top-k then softmax, 2 sigmoid scores with a
// selection bias (sel_b, may be null), optional renormalisation and a scale
int launch_moe_topk(const swarm::GemmOut& lg, const float* br, int T, int E, int k, int mode,
                    const float* sel_b, int norm, float scale, int32_t* ids, float* wts,
                    int* counts, cudaStream_t s);
int launch_moe_plan(int* counts, int E, int tok_tile, int* offsets, int* cursor, void* tiles,
                    int* n_tiles, int max_tiles, int* status, cudaStream_t s);
int launch_moe_scatter(const __half* x, int x_stride, int H, const int32_t* ids, int P, int k,
                       int* cursor, void* xs, int xs_stride, int xs_bf16, int32_t* ret,
                       int rank, cudaStream_t s);
int launch_moe_gemm_tc(int fmt, int epi, const void* w, int rows, int K, const void* xs,
                       int xs_stride, int xs_rows, int tok_tile, const void* tiles,
                       const int* n_tiles, int max_tiles, const float* bias, int bias_stride,
                       void* h, int h_stride, int act_kind, float alpha, float limit,
                       const unsigned long long* out_ptrs, int n_out, int out_stride,
                       const int32_t* ret, int num_sms, int* status, cudaStream_t s,
                       int* sig_ctl = nullptr, const unsigned long long* sig_bases = nullptr,
                       long long sig_flag_off = 0, int sig_world = 0, int sig_rank = 0);
int launch_moe_combine(const float* rows, int row_stride, const float* wts, int k,
                       const swarm::GemmOut* sh, const swarm::GemmOut* shg, float* residual,
                       int T, int H, const float* norm_w, __half* out, int out_stride, float eps,
                       cudaStream_t s);

// Tensor parallelism over the experts (every rank: every token, experts [e0, e0+n_loc)).
int launch_moe_localize(int32_t* ids, float* wts, int* counts, int P, int E, int e0, int n_loc,
                        cudaStream_t s);
int launch_moe_combine_tp(const float* rows, int row_stride, const float* wts, int k,
                          const swarm::GemmOut* sh, const swarm::GemmOut* shg, int T, int H, int W,
                          const unsigned long long* dst, int* ctl, const unsigned long long* bases,
                          long long flag_off, int rank, cudaStream_t s, int to_all = 0);

void launch_mul_f16(__half* x, const __half* y, size_t n, cudaStream_t s);

// ---- gated DeltaNet (deltanet.cu) --------------------------------------------
// seqs: int32 [S][4] = (row0, nrows, state slot, position of row0)
int launch_ssm_conv_silu(const swarm::GemmOut& g, const float* w, int C, int K, float* state,
                         const void* seqs, int S, float* out, cudaStream_t s);
int launch_delta_rule(const float* qkv, int C, int nk, int nv, int D, const swarm::GemmOut& gba,
                      const float* dt_bias, const float* A, const swarm::GemmOut& gz,
                      const float* norm_w, float eps, float* state, const void* seqs, int S,
                      __half* out, cudaStream_t s);
int launch_delta_chunk(const float* qkv, int C, int nk, int nv, int D, const swarm::GemmOut& gba,
                       const float* dt_bias, const float* A, const swarm::GemmOut& gz,
                       const float* norm_w, float eps, float* state, const void* seqs, int S,
                       int T, float* o_raw, __half* out, cudaStream_t s);

// ---- expert parallelism over peer memory (ep_comm.cu) --------------------------
long long ep_arena_bytes(int world, int cap, int H, int e_loc);
void ep_arena_offsets(int world, int cap, int H, int e_loc, long long* out6);
int ep_arena_alloc(long long bytes, void** ptr, void* handle64);
int ep_arena_open(const void* handle64, void** ptr);
int ep_arena_close(void* ptr, int own);
int launch_ep_dispatch(const __half* x, int x_stride, int H, const int32_t* ids, int P, int k,
                       int* counts, int E, int e_loc, int cap, int* cursor,
                       const unsigned long long* bases, int world, int rank, int x_bf16,
                       int* ctl, cudaStream_t s);
int launch_ep_wait(unsigned long long own_base, int world, int cap, int H, int e_loc, int which,
                   int* ctl, int* status, cudaStream_t s, long long timeout_ns = 0);
int launch_ep_plan_owner(unsigned long long own_base, int world, int cap, int H, int e_loc,
                         int tok_tile, void* tiles, int* n_tiles, int max_tiles, int* status,
                         cudaStream_t s);

// ---- speculative tree ranking (tree_rank.cu) ---------------------------------
int tree_rank_slices(int rows, int V);
int launch_tree_rank(const float* logits, int rows, int V, int stride, int k, float* cand_v,
                     int* cand_i, float* ms, int S, int32_t* ids, float* logp, cudaStream_t s);
// Bounded wait (one CTA) until flags[0..world) reach this side's next epoch
// (ctl[slot] + 1); records code/where in status on timeout.
// Tensor parallelism (tp_comm.cu): reduce of the owner-routed partials + residual
// + RMSNorm + all-gather of the residual over peer memory.
int tp_reduce_slices(int T, int H, int W, int num_sms);  // CTAs per row of tp_reduce_norm
int launch_tp_reduce_norm(const swarm::GemmOut& g, const float* bias, const float* w, __half* out,
                          int out_stride, float eps, int H, int W, int rank, int T, int t_stride,
                          const unsigned long long* bases, long long h_in_off, long long h_out_off,
                          long long ss_off, long long rowflag_off, const void* gemm_flags,
                          int* ctl_gemm, int* ctl_row, int* status, int code, int num_sms,
                          long long timeout_ns, cudaStream_t s);
int launch_flag_wait(const void* flags, int world, int* ctl, int slot, int* status, int code,
                     cudaStream_t s, long long timeout_ns = 0);
// One-hop TP reduce for few rows: every rank received every rank's partials
// (GemmOut n_src = W); wait for the W GEMM-done flags, then residual += sum
// (+ bias) in place and out = RMSNorm(residual) * w (w / out may be null).
int launch_tp_local_norm(const swarm::GemmOut& g, float* residual, const float* bias,
                         const float* w, __half* out, int out_stride, float eps, int W,
                         const void* gemm_flags, int* ctl_gemm, int* ctl_done, int* status,
                         int code, long long timeout_ns, cudaStream_t s);

// Diagnostics (mma_probe.cu): clock64 cycles of `iters` x 4 back-to-back
// tcgen05.mma of probe shape `shape` (every `group` MMAs, when group > 0: a
// commit, with a wait if mode & 1, or a `spin`-clock pause if mode & 4; mode
// & 2 rotates over 4 accumulators), one entry per CTA.
int mma_probe_shapes();
void mma_probe_shape(int i, int* ts, int* m, int* n);
int launch_mma_probe(int shape, int iters, int group, int mode, int spin, int ctas,
                     long long* cycles, cudaStream_t s);

// GGML blocks -> fp16 [rows][K] (qmatmul_simt.cu); quantized types only.
int launch_dequant_f16(const void* w, int type, int rows, int K, __half* out, cudaStream_t s);

// ---- LoRA (lora.cu) -----------------------------------------------------------
int launch_lora(const __half* x, int x_stride, int K, const int32_t* ids, int T, const __half* A,
                const __half* B, const float* scale, int R, int rows, float* u, float* delta,
                cudaStream_t s);
