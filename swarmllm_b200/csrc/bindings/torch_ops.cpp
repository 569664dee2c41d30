// PyTorch bindings for the sm_100a kernels (module swarmllm_b200._C).
// Every op launches on torch's current CUDA stream, so they can be captured in
// CUDA graphs.  Shapes and dtypes are checked here; the kernels trust them.
#include "ops_common.h"

// ---------------------------------------------------------------- elementwise
void embed_gather(Tensor table, int64_t type, int64_t hidden, Tensor ids, Tensor out) {
  CHECK_CUDA(table); CHECK_CUDA(ids); CHECK_CUDA(out);
  CHECK_DT(ids, at::kInt); CHECK_DT(out, at::kFloat);
  const at::cuda::CUDAGuard guard(out.device());
  launch_embed_gather(table.data_ptr(), (int)type, (int)hidden, ids.data_ptr<int32_t>(),
                      (int)ids.numel(), out.data_ptr<float>(), cur_stream());
}

void rmsnorm(Tensor x, Tensor w, Tensor out, double eps) {
  CHECK_CUDA(x); CHECK_DT(x, at::kFloat); CHECK_DT(w, at::kFloat); CHECK_DT(out, at::kHalf);
  CHECK_CONTIG(x); CHECK_CONTIG(out);
  const at::cuda::CUDAGuard guard(x.device());
  const int dim = (int)x.size(-1);
  launch_rmsnorm(x.data_ptr<float>(), w.data_ptr<float>(),
                 reinterpret_cast<__half*>(out.data_ptr()), (int)(x.numel() / dim), dim,
                 (float)eps, cur_stream());
}

void epi_residual_rmsnorm(const GemmResult& g, Tensor residual, OptT bias, Tensor w, OptT out,
                          double eps, OptT post_w) {
  CHECK_DT(residual, at::kFloat);
  TORCH_CHECK(residual.size(-1) == g.g.rows, "residual width != GEMM rows");
  const at::cuda::CUDAGuard guard(residual.device());
  launch_epi_residual_rmsnorm(g.g, residual.data_ptr<float>(), ptr_or_null<float>(bias),
                              w.data_ptr<float>(), ptr_or_null<__half>(out), (float)eps,
                              out.has_value() ? (int)out->stride(0) : 0, cur_stream(),
                              ptr_or_null<float>(post_w));
}

void epi_rope_kv(const GemmResult& g, OptT bias, Tensor positions, OptT slots, Tensor inv_freq,
                 int64_t n_q, int64_t n_kv, int64_t head_dim, int64_t rope_dim, bool neox,
                 double attn_factor, Tensor q_out, OptT k_cache, OptT v_cache, int64_t page_size,
                 OptT q_norm_w, OptT k_norm_w, double norm_eps, OptT gate_out) {
  CHECK_DT(positions, at::kInt); CHECK_DT(q_out, at::kHalf); CHECK_DT(inv_freq, at::kFloat);
  TORCH_CHECK(g.g.rows == (n_q * (gate_out.has_value() ? 2 : 1) + 2 * n_kv) * head_dim,
              "QKV rows mismatch");
  TORCH_CHECK(head_dim % 4 == 0 && rope_dim % 2 == 0 && rope_dim <= head_dim,
              "head_dim must be a multiple of 4 and rope_dim even");
  const at::cuda::CUDAGuard guard(q_out.device());
  launch_epi_rope_kv(g.g, ptr_or_null<float>(bias), positions.data_ptr<int32_t>(),
                     ptr_or_null<int32_t>(slots), inv_freq.data_ptr<float>(), (int)n_q, (int)n_kv,
                     (int)head_dim, (int)rope_dim, neox ? 1 : 0, (float)attn_factor,
                     reinterpret_cast<__half*>(q_out.data_ptr()), ptr_or_null<__half>(k_cache),
                     ptr_or_null<__half>(v_cache), (int)page_size, ptr_or_null<float>(q_norm_w),
                     ptr_or_null<float>(k_norm_w), (float)norm_eps, ptr_or_null<__half>(gate_out),
                     cur_stream());
}

void epi_swiglu(const GemmResult& g, OptT bias, int64_t F, int64_t kind, bool interleaved,
                double alpha, double limit, Tensor out) {
  CHECK_DT(out, at::kHalf);
  TORCH_CHECK(g.g.rows == 2 * F, "gate_up rows must be 2F");
  const at::cuda::CUDAGuard guard(out.device());
  launch_epi_swiglu(g.g, ptr_or_null<float>(bias), (int)F, (int)kind, interleaved ? 1 : 0,
                    (float)alpha, (float)limit, reinterpret_cast<__half*>(out.data_ptr()),
                    cur_stream());
}

void epi_copy(const GemmResult& g, OptT bias, Tensor out) {
  CHECK_DT(out, at::kFloat);
  const at::cuda::CUDAGuard guard(out.device());
  launch_epi_copy(g.g, ptr_or_null<float>(bias), out.data_ptr<float>(), (int)out.stride(0),
                  cur_stream());
}

// ---------------------------------------------------------------- GEMMs
GemmResult qmatmul_simt(Tensor w, int64_t type, int64_t rows, int64_t K, Tensor x, Tensor out) {
  CHECK_CUDA(w); CHECK_CUDA(x); CHECK_DT(x, at::kHalf); CHECK_DT(out, at::kFloat);
  TORCH_CHECK(x.size(-1) == K && x.stride(-1) == 1, "x must be [T, K] with unit inner stride");
  TORCH_CHECK(out.size(-1) == rows && out.is_contiguous(), "out must be [T, rows] contiguous");
  const at::cuda::CUDAGuard guard(x.device());
  const int T = (int)x.size(0);
  int rc = launch_qmatmul_simt(w.data_ptr(), (int)type, (int)rows, (int)K,
                               reinterpret_cast<const __half*>(x.data_ptr()), (int)x.stride(0), T,
                               out.data_ptr<float>(), (int)rows, cur_stream());
  TORCH_CHECK(rc == 0, "qmatmul_simt: unsupported type ", type);
  GemmResult r;
  r.g.ws = out.data_ptr<float>();
  r.g.rows = (int)rows;
  r.g.T = T;
  r.g.mode = 0;
  r.ws = out;
  return r;
}

py::tuple q4k_tc_plan_py(int64_t rows, int64_t K, int64_t T, int64_t num_sms, int64_t fmt) {
  int N, ntt, kb, upc, ctas;
  long total;
  size_t need;
  q4k_tc_plan((int)rows, (int)K, (int)T, (int)num_sms, &N, &ntt, &kb, &total, &upc, &ctas, &need,
              (int)fmt);
  return py::make_tuple(N, ntt, kb, total, upc, ctas, need);
}

GemmResult qgemm_q4k_tc(Tensor w_packed, int64_t rows, int64_t K, Tensor x, Tensor ws,
                        Tensor status, int64_t num_sms, int64_t fmt, OptT w_b, int64_t fmt_b,
                        int64_t split_tile) {
  CHECK_CUDA(w_packed); CHECK_CUDA(x); CHECK_DT(x, at::kHalf); CHECK_DT(ws, at::kFloat);
  CHECK_DT(status, at::kInt);
  TORCH_CHECK(status.numel() >= 8, "status must hold 8 ints");
  TORCH_CHECK(x.size(-1) == K && x.stride(-1) == 1, "x must be [T, K] with unit inner stride");
  const at::cuda::CUDAGuard guard(x.device());
  const int T = (int)x.size(0);
  if (num_sms <= 0) num_sms = num_sms_of(x);
  GemmResult r;
  int rc = launch_qgemm_q4k_tc(w_packed.data_ptr(), (int)rows, (int)K,
                               reinterpret_cast<const __half*>(x.data_ptr()), (int)x.stride(0), T,
                               ws.data_ptr<float>(), (size_t)ws.numel(), (int)num_sms,
                               status.data_ptr<int>(), &r.g, cur_stream(), nullptr, 0, nullptr,
                               nullptr, 0, 0, 0, (int)fmt, ptr_or_null<void>(w_b),
                               w_b.has_value() ? (int)fmt_b : -1, (int)split_tile);
  TORCH_CHECK(rc == 0, "qgemm_q4k_tc launch failed: rc=", rc);
  r.ws = ws;
  return r;
}

GemmResult dense_gemm_tc(Tensor w, Tensor x, Tensor ws, Tensor status, int64_t num_sms) {
  CHECK_DT(w, at::kHalf); CHECK_DT(x, at::kHalf); CHECK_DT(ws, at::kFloat);
  CHECK_DT(status, at::kInt);
  TORCH_CHECK(status.numel() >= 8, "status must hold 8 ints");
  TORCH_CHECK(w.dim() == 2 && w.stride(1) == 1 && x.stride(-1) == 1, "row-major operands");
  TORCH_CHECK(x.size(-1) == w.size(1), "K mismatch");
  const at::cuda::CUDAGuard guard(x.device());
  if (num_sms <= 0) num_sms = num_sms_of(x);
  GemmResult r;
  int rc = launch_dense_gemm_tc(reinterpret_cast<const __half*>(w.data_ptr()), (int)w.size(0),
                                (int)w.size(1), (int)w.stride(0),
                                reinterpret_cast<const __half*>(x.data_ptr()), (int)x.stride(0),
                                (int)x.size(0), ws.data_ptr<float>(), (size_t)ws.numel(),
                                (int)num_sms, status.data_ptr<int>(), &r.g, cur_stream());
  TORCH_CHECK(rc == 0, "dense_gemm_tc launch failed: rc=", rc);
  r.ws = ws;
  return r;
}

py::tuple dense_tc_plan_py(int64_t rows, int64_t K, int64_t T, int64_t num_sms) {
  int N, ntt, kb, upc, ctas;
  long total;
  size_t need;
  dense_tc_plan((int)rows, (int)K, (int)T, (int)num_sms, &N, &ntt, &kb, &total, &upc, &ctas, &need);
  return py::make_tuple(N, ntt, kb, total, upc, ctas, need);
}

// Row-parallel Q4_K GEMM of a tensor-parallel group: partial tiles pushed to
// every rank's receive buffer (dst_ptrs[o]); the result reads this rank's
// receive buffer, summing the n ranks' partials (src_stride floats apart).
GemmResult qgemm_q4k_tc_tp(Tensor w_packed, int64_t rows, int64_t K, Tensor x, Tensor status,
                           int64_t num_sms, int64_t recv_base, int64_t src_stride,
                           std::vector<int64_t> dst_ptrs, Tensor sig_ctl,
                           std::vector<int64_t> sig_bases, int64_t sig_flag_off, int64_t rank,
                           int64_t owner_tiles, int64_t fmt) {
  CHECK_CUDA(w_packed); CHECK_DT(x, at::kHalf); CHECK_DT(status, at::kInt);
  CHECK_DT(sig_ctl, at::kInt);
  TORCH_CHECK(x.size(-1) == K && x.stride(-1) == 1, "x must be [T, K] with unit inner stride");
  TORCH_CHECK(dst_ptrs.size() == sig_bases.size() && !dst_ptrs.empty() && dst_ptrs.size() <= 8,
              "1..8 ranks");
  const at::cuda::CUDAGuard guard(x.device());
  if (num_sms <= 0) num_sms = num_sms_of(x);
  unsigned long long d[8], b[8];
  for (size_t i = 0; i < dst_ptrs.size(); ++i) {
    d[i] = (unsigned long long)dst_ptrs[i];
    b[i] = (unsigned long long)sig_bases[i];
  }
  GemmResult r;
  float* own = reinterpret_cast<float*>(recv_base);
  int rc = launch_qgemm_q4k_tc(w_packed.data_ptr(), (int)rows, (int)K,
                               reinterpret_cast<const __half*>(x.data_ptr()), (int)x.stride(0),
                               (int)x.size(0), own, (size_t)src_stride, (int)num_sms,
                               status.data_ptr<int>(), &r.g, cur_stream(), d,
                               (int)dst_ptrs.size(), sig_ctl.data_ptr<int>(), b,
                               (long long)sig_flag_off, (int)rank, (int)owner_tiles, (int)fmt);
  TORCH_CHECK(rc == 0, "qgemm_q4k_tc_tp launch failed: rc=", rc);
  r.g.n_src = (int)dst_ptrs.size();
  r.g.src_stride = src_stride;
  return r;
}

// Fused TP reduction of a row-parallel GEMM's owner-routed partials + residual
// + RMSNorm + residual all-gather (tp_comm.cu).  Offsets are bytes into every
// rank's arena (same layout on all ranks).
void tp_reduce_norm(const GemmResult& g, OptT bias, OptT w, OptT out, double eps, int64_t H,
                    int64_t rank, int64_t T, int64_t t_stride, std::vector<int64_t> bases,
                    int64_t h_in_off, int64_t h_out_off, int64_t ss_off, int64_t rowflag_off,
                    int64_t gemm_flags, Tensor ctl, int64_t ctl_gemm_slot, int64_t ctl_row_slot,
                    Tensor status, int64_t code, int64_t num_sms, int64_t timeout_ns) {
  CHECK_DT(ctl, at::kInt); CHECK_DT(status, at::kInt);
  TORCH_CHECK(!bases.empty() && bases.size() <= 8, "1..8 ranks");
  if (out.has_value()) CHECK_DT(*out, at::kHalf);
  const at::cuda::CUDAGuard guard(ctl.device());
  unsigned long long b[8];
  for (size_t i = 0; i < bases.size(); ++i) b[i] = (unsigned long long)bases[i];
  int* c = ctl.data_ptr<int>();
  int rc = launch_tp_reduce_norm(
      g.g, ptr_or_null<float>(bias), ptr_or_null<float>(w), ptr_or_null<__half>(out),
      out.has_value() ? (int)out->stride(0) : 0, (float)eps, (int)H, (int)bases.size(), (int)rank,
      (int)T, (int)t_stride, b, h_in_off, h_out_off, ss_off, rowflag_off,
      reinterpret_cast<const void*>(gemm_flags), c + ctl_gemm_slot, c + ctl_row_slot,
      status.data_ptr<int>(), (int)code, (int)num_sms, (long long)timeout_ns, cur_stream());
  TORCH_CHECK(rc == 0, "tp_reduce_norm launch failed: rc=", rc);
}

// One-hop TP reduce for few rows (tp_comm.cu tp_local_norm_kernel).
void tp_local_norm(const GemmResult& g, Tensor residual, OptT bias, OptT w, OptT out, double eps,
                   int64_t W, int64_t gemm_flags, Tensor ctl, int64_t ctl_gemm_slot,
                   int64_t ctl_done_slot, Tensor status, int64_t code, int64_t timeout_ns) {
  CHECK_DT(residual, at::kFloat); CHECK_DT(ctl, at::kInt); CHECK_DT(status, at::kInt);
  TORCH_CHECK(residual.size(-1) == g.g.rows && residual.size(0) >= g.g.T, "residual shape");
  if (out.has_value()) CHECK_DT(*out, at::kHalf);
  const at::cuda::CUDAGuard guard(ctl.device());
  int* c = ctl.data_ptr<int>();
  int rc = launch_tp_local_norm(g.g, residual.data_ptr<float>(), ptr_or_null<float>(bias),
                                ptr_or_null<float>(w), ptr_or_null<__half>(out),
                                out.has_value() ? (int)out->stride(0) : 0, (float)eps, (int)W,
                                reinterpret_cast<const void*>(gemm_flags), c + ctl_gemm_slot,
                                c + ctl_done_slot, status.data_ptr<int>(), (int)code,
                                (long long)timeout_ns, cur_stream());
  TORCH_CHECK(rc == 0, "tp_local_norm launch failed: rc=", rc);
}

void qgemm_set_trace_py(OptT buf) {
  if (buf.has_value()) TORCH_CHECK(buf->numel() * buf->element_size() >= 512 * 8 * 8, "trace buffer too small");
  qgemm_set_trace(ptr_or_null<void>(buf));
}

void q4k_repack(Tensor src, int64_t rows, int64_t K, Tensor dst) {
  CHECK_CUDA(src); CHECK_CUDA(dst);
  TORCH_CHECK(K % 256 == 0, "K must be a multiple of 256");
  const int64_t rows_pad = (rows + 127) / 128 * 128;
  TORCH_CHECK(dst.numel() * dst.element_size() >= rows_pad * (K / 256) * 144, "dst too small");
  const at::cuda::CUDAGuard guard(dst.device());
  TORCH_CHECK(launch_q4k_repack(src.data_ptr(), (int)rows, (int)K, dst.data_ptr(), cur_stream()) == 0,
              "repack launch failed");
}

// GGUF Q4_K / Q6_K / Q8_0 rows -> the tiled layout of format `fmt` (qfmt.cuh).
void qfmt_repack(int64_t fmt, Tensor src, int64_t rows, int64_t K, Tensor dst) {
  CHECK_CUDA(src); CHECK_CUDA(dst);
  TORCH_CHECK(fmt >= 0 && fmt <= 2, "unknown format");
  TORCH_CHECK(K % 256 == 0, "K must be a multiple of 256");
  const int64_t rows_pad = (rows + 127) / 128 * 128;
  TORCH_CHECK(dst.numel() * dst.element_size() >= rows_pad * (K / 256) * qfmt_row_bytes((int)fmt),
              "dst too small");
  const at::cuda::CUDAGuard guard(dst.device());
  TORCH_CHECK(launch_qfmt_repack((int)fmt, src.data_ptr(), (int)rows, (int)K, dst.data_ptr(),
                                 cur_stream()) == 0,
              "repack launch failed");
}

// ---------------------------------------------------------------- attention
void decode_attn(Tensor q, Tensor k_cache, Tensor v_cache, Tensor block_table, Tensor seq_lens,
                 OptT tree_mask, OptT tree_start, OptT sinks, int64_t window, double scale,
                 double softcap, int64_t keys_per_split, Tensor part_o, Tensor part_ml,
                 Tensor out) {
  CHECK_DT(q, at::kHalf); CHECK_DT(k_cache, at::kHalf); CHECK_DT(v_cache, at::kHalf);
  CHECK_DT(block_table, at::kInt); CHECK_DT(seq_lens, at::kInt); CHECK_DT(out, at::kHalf);
  CHECK_CONTIG(q); CHECK_CONTIG(out); CHECK_CONTIG(block_table);
  const at::cuda::CUDAGuard guard(q.device());
  const int T = (int)q.size(0), n_q = (int)q.size(1), d = (int)q.size(2);
  const int n_kv = (int)k_cache.size(1), page = (int)k_cache.size(2);
  const int n_splits = (int)part_ml.size(2);
  TORCH_CHECK(part_o.size(2) == n_splits && part_o.size(3) == d, "part_o shape");
  int rc = launch_decode_attn_simt(
      reinterpret_cast<const __half*>(q.data_ptr()),
      reinterpret_cast<const __half*>(k_cache.data_ptr()),
      reinterpret_cast<const __half*>(v_cache.data_ptr()), block_table.data_ptr<int32_t>(),
      (int)block_table.stride(0), seq_lens.data_ptr<int32_t>(),
      ptr_or_null<uint64_t>(tree_mask), ptr_or_null<int32_t>(tree_start), ptr_or_null<float>(sinks),
      T, n_q, n_kv, d, page, (int)window, (float)scale, (float)softcap, (int)keys_per_split,
      n_splits, part_o.data_ptr<float>(), part_ml.data_ptr<float>(),
      reinterpret_cast<__half*>(out.data_ptr()), cur_stream());
  TORCH_CHECK(rc == 0, "decode_attn: unsupported head_dim/group size");
}

void attn_tc(Tensor q, Tensor k_cache, Tensor v_cache, Tensor group_row0, Tensor group_npos,
             int64_t pos_per_group, Tensor block_table, Tensor seq_lens, OptT tree_mask,
             OptT tree_start, OptT sinks, int64_t window, double scale, int64_t keys_per_split,
             int64_t n_splits, Tensor out, Tensor part_o, Tensor part_ml, Tensor status) {
  CHECK_DT(q, at::kHalf); CHECK_DT(k_cache, at::kHalf); CHECK_DT(v_cache, at::kHalf);
  CHECK_DT(block_table, at::kInt); CHECK_DT(seq_lens, at::kInt); CHECK_DT(out, at::kHalf);
  CHECK_DT(group_row0, at::kInt); CHECK_DT(group_npos, at::kInt); CHECK_DT(status, at::kInt);
  CHECK_CONTIG(q); CHECK_CONTIG(out); CHECK_CONTIG(block_table); CHECK_CONTIG(k_cache);
  TORCH_CHECK(status.numel() >= 8, "status must hold 8 ints");
  const at::cuda::CUDAGuard guard(q.device());
  const int T = (int)q.size(0), n_q = (int)q.size(1), d = (int)q.size(2);
  const int n_kv = (int)k_cache.size(1);
  TORCH_CHECK(k_cache.size(2) == 16 && k_cache.size(3) == d, "cache must be [pages, n_kv, 16, d]");
  const int G = (int)group_row0.numel();
  int rc = launch_attn_tc(
      reinterpret_cast<const __half*>(q.data_ptr()), T, n_q,
      reinterpret_cast<const __half*>(k_cache.data_ptr()),
      reinterpret_cast<const __half*>(v_cache.data_ptr()), (long)k_cache.size(0), n_kv, d,
      group_row0.data_ptr<int32_t>(), group_npos.data_ptr<int32_t>(), G, (int)pos_per_group,
      block_table.data_ptr<int32_t>(), (int)block_table.stride(0), seq_lens.data_ptr<int32_t>(),
      ptr_or_null<uint64_t>(tree_mask), ptr_or_null<int32_t>(tree_start), ptr_or_null<float>(sinks),
      (int)window, (float)scale, (int)keys_per_split, (int)n_splits,
      reinterpret_cast<__half*>(out.data_ptr()), part_o.data_ptr<float>(), part_ml.data_ptr<float>(),
      status.data_ptr<int>(), cur_stream());
  TORCH_CHECK(rc == 0, "attn_tc launch failed: rc=", rc);
  if (n_splits > 1)
    launch_attn_combine(part_o.data_ptr<float>(), part_ml.data_ptr<float>(), T * n_q, (int)n_splits,
                        d, ptr_or_null<float>(sinks), n_q, reinterpret_cast<__half*>(out.data_ptr()),
                        cur_stream());
}

// ---------------------------------------------------------------- sampling
void argmax(Tensor logits, Tensor out, OptT out_val) {
  CHECK_DT(logits, at::kFloat); CHECK_DT(out, at::kInt);
  const at::cuda::CUDAGuard guard(logits.device());
  launch_argmax(logits.data_ptr<float>(), (int)logits.size(0), (int)logits.size(1),
                (int)logits.stride(0), out.data_ptr<int32_t>(), ptr_or_null<float>(out_val),
                cur_stream());
}

void sample(Tensor logits, Tensor temperature, OptT top_k, OptT top_p, OptT seeds, OptT positions,
            Tensor out) {
  CHECK_DT(logits, at::kFloat); CHECK_DT(out, at::kInt); CHECK_DT(temperature, at::kFloat);
  const at::cuda::CUDAGuard guard(logits.device());
  launch_sample(logits.data_ptr<float>(), (int)logits.size(0), (int)logits.size(1),
                (int)logits.stride(0), temperature.data_ptr<float>(), ptr_or_null<int32_t>(top_k),
                ptr_or_null<float>(top_p), ptr_or_null<uint64_t>(seeds),
                ptr_or_null<int32_t>(positions), out.data_ptr<int32_t>(), cur_stream());
}

void apply_penalties(Tensor logits, Tensor off, Tensor tok, Tensor val) {
  CHECK_DT(logits, at::kFloat); CHECK_DT(off, at::kInt); CHECK_DT(tok, at::kInt);
  CHECK_DT(val, at::kFloat);
  TORCH_CHECK(off.numel() == logits.size(0) + 1 && tok.numel() == val.numel(),
              "penalty table shape");
  const at::cuda::CUDAGuard guard(logits.device());
  launch_apply_penalties(logits.data_ptr<float>(), (int)logits.size(0), (int)logits.size(1),
                         (int)logits.stride(0), off.data_ptr<int32_t>(), tok.data_ptr<int32_t>(),
                         val.data_ptr<float>(), cur_stream());
}

void philox_uniform(int64_t seed, Tensor positions, int64_t V, Tensor out) {
  const at::cuda::CUDAGuard guard(out.device());
  launch_philox_uniform((uint64_t)seed, positions.data_ptr<int32_t>(), (int)positions.numel(),
                        (int)V, out.data_ptr<float>(), cur_stream());
}

// SWARMLLM_SEGV_BT=1: print a native backtrace on SIGSEGV (debug aid for
// host-side crashes; there is no debugger on the GPU boxes).
static void segv_handler(int sig) {
  void* frames[64];
  int n = backtrace(frames, 64);
  const char msg[] = "\n[swarmllm] native backtrace:\n";
  (void)!write(2, msg, sizeof(msg) - 1);
  backtrace_symbols_fd(frames, n, 2);
  signal(sig, SIG_DFL);
  raise(sig);
}

void register_moe_ops(py::module& m);
void register_ep_ops(py::module& m);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "swarmllm_b200 sm_100a kernels";
  if (const char* e = getenv("SWARMLLM_SEGV_BT")) {
    if (e[0] == '1') signal(SIGSEGV, segv_handler);
  }
  py::class_<GemmResult>(m, "GemmResult")
      .def_property_readonly("rows", [](const GemmResult& r) { return r.g.rows; })
      .def_property_readonly("T", [](const GemmResult& r) { return r.g.T; })
      .def_property_readonly("mode", [](const GemmResult& r) { return r.g.mode; })
      .def_property_readonly("tok_tile", [](const GemmResult& r) { return r.g.tok_tile; })
      .def_property_readonly("upc", [](const GemmResult& r) { return r.g.upc; })
      .def_property_readonly("ksb", [](const GemmResult& r) { return r.g.ksb; })
      .def_readonly("ws", &GemmResult::ws);
  m.def("embed_gather", &embed_gather);
  m.def("rmsnorm", &rmsnorm);
  m.def("epi_residual_rmsnorm", &epi_residual_rmsnorm, py::arg("g"), py::arg("residual"),
        py::arg("bias"), py::arg("w"), py::arg("out"), py::arg("eps"),
        py::arg("post_w") = py::none());
  m.def("epi_rope_kv", &epi_rope_kv, py::arg("g"), py::arg("bias"), py::arg("positions"),
        py::arg("slots"), py::arg("inv_freq"), py::arg("n_q"), py::arg("n_kv"),
        py::arg("head_dim"), py::arg("rope_dim"), py::arg("neox"), py::arg("attn_factor"),
        py::arg("q_out"), py::arg("k_cache"), py::arg("v_cache"), py::arg("page_size"),
        py::arg("q_norm_w"), py::arg("k_norm_w"), py::arg("norm_eps"),
        py::arg("gate_out") = py::none());
  m.def("mul_f16", [](Tensor x, Tensor y) {
    CHECK_DT(x, at::kHalf); CHECK_DT(y, at::kHalf); CHECK_CONTIG(x); CHECK_CONTIG(y);
    TORCH_CHECK(x.numel() == y.numel(), "size mismatch");
    const at::cuda::CUDAGuard guard(x.device());
    launch_mul_f16(reinterpret_cast<__half*>(x.data_ptr()),
                   reinterpret_cast<const __half*>(y.data_ptr()), (size_t)x.numel(), cur_stream());
  });
  m.def("ssm_conv_silu", [](const GemmResult& g, Tensor w, Tensor state, Tensor seqs, int64_t S,
                            Tensor out) {
    CHECK_DT(w, at::kFloat); CHECK_DT(state, at::kFloat); CHECK_DT(seqs, at::kInt);
    CHECK_DT(out, at::kFloat); CHECK_CONTIG(w); CHECK_CONTIG(out);
    TORCH_CHECK(w.dim() == 2 && w.size(0) == g.g.rows, "conv weight [C, K]");
    TORCH_CHECK(out.size(-1) == g.g.rows, "out width");
    const at::cuda::CUDAGuard guard(out.device());
    int rc = launch_ssm_conv_silu(g.g, w.data_ptr<float>(), (int)w.size(0), (int)w.size(1),
                                  state.data_ptr<float>(), seqs.data_ptr(), (int)S,
                                  out.data_ptr<float>(), cur_stream());
    TORCH_CHECK(rc == 0, "ssm_conv_silu failed: rc=", rc);
  });
  m.def("lora_delta", [](Tensor x, Tensor ids, Tensor A, Tensor B, Tensor scale, Tensor u,
                         Tensor delta) {
    // x [T, K] fp16, ids [T] int32, A [M, R, K] fp16, B [M, rows, R] fp16, scale [M] fp32,
    // u >= [T, R] fp32 scratch, delta [T, rows] fp32 (out)
    CHECK_DT(x, at::kHalf); CHECK_DT(ids, at::kInt); CHECK_DT(A, at::kHalf); CHECK_DT(B, at::kHalf);
    CHECK_DT(scale, at::kFloat); CHECK_DT(u, at::kFloat); CHECK_DT(delta, at::kFloat);
    CHECK_CONTIG(A); CHECK_CONTIG(B); CHECK_CONTIG(delta);
    const int T = (int)x.size(0), K = (int)x.size(1), R = (int)A.size(1), rows = (int)B.size(1);
    TORCH_CHECK(A.size(2) == K && B.size(2) == R && u.numel() >= (int64_t)T * R &&
                delta.size(0) >= T && delta.size(1) == rows, "lora shapes");
    const at::cuda::CUDAGuard guard(x.device());
    TORCH_CHECK(launch_lora(reinterpret_cast<const __half*>(x.data_ptr()), (int)x.stride(0), K,
                            ids.data_ptr<int32_t>(), T,
                            reinterpret_cast<const __half*>(A.data_ptr()),
                            reinterpret_cast<const __half*>(B.data_ptr()), scale.data_ptr<float>(),
                            R, rows, u.data_ptr<float>(), delta.data_ptr<float>(), cur_stream()) == 0,
                "lora launch failed");
  });
  m.def("dequant_f16", [](Tensor raw, int64_t qtype, int64_t rows, int64_t K, Tensor out) {
    CHECK_CUDA(raw); CHECK_DT(out, at::kHalf); CHECK_CONTIG(out);
    TORCH_CHECK(out.numel() >= rows * K, "out too small");
    const at::cuda::CUDAGuard guard(raw.device());
    const int rc = launch_dequant_f16(raw.data_ptr(), (int)qtype, (int)rows, (int)K,
                                      reinterpret_cast<__half*>(out.data_ptr()), cur_stream());
    TORCH_CHECK(rc == 0, "dequant_f16 failed: rc=", rc);
  });
  m.def("gemm_with_add", [](const GemmResult& g, Tensor add) {
    CHECK_DT(add, at::kFloat);
    TORCH_CHECK(add.size(-1) == g.g.rows && add.stride(-1) == 1, "add must be [T, rows]");
    GemmResult r = g;
    r.g.add = add.data_ptr<float>();
    r.g.add_stride = (int)add.stride(0);
    return r;
  });
  m.def("tree_rank", [](Tensor logits, int64_t k, Tensor ids, Tensor logp, Tensor ws) {
    // ws: float32 scratch of at least rows * S * (2k + 2) elements (tree_rank_ws_floats)
    CHECK_DT(logits, at::kFloat); CHECK_DT(ids, at::kInt); CHECK_DT(logp, at::kFloat);
    CHECK_DT(ws, at::kFloat);
    TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "logits [rows, V] row-major");
    const int rows = (int)logits.size(0), V = (int)logits.size(1);
    TORCH_CHECK(ids.numel() >= rows * k && logp.numel() >= rows * k, "outputs too small");
    const int S = tree_rank_slices(rows, V);
    TORCH_CHECK(ws.numel() >= (int64_t)rows * S * (2 * k + 2), "tree_rank workspace too small");
    const at::cuda::CUDAGuard guard(logits.device());
    float* base = ws.data_ptr<float>();
    int rc = launch_tree_rank(logits.data_ptr<float>(), rows, V, (int)logits.stride(0), (int)k,
                              base, reinterpret_cast<int*>(base + (size_t)rows * S * k),
                              base + (size_t)rows * S * 2 * k, S, ids.data_ptr<int32_t>(),
                              logp.data_ptr<float>(), cur_stream());
    TORCH_CHECK(rc == 0, "tree_rank failed: rc=", rc);
  });
  m.def("tree_rank_ws_floats", [](int64_t rows, int64_t V, int64_t k) {
    return (int64_t)rows * tree_rank_slices((int)rows, (int)V) * (2 * k + 2);
  });
  m.def("delta_chunk", [](Tensor qkv, int64_t nk, int64_t nv, int64_t D, const GemmResult& gba,
                          Tensor dt_bias, Tensor A, const GemmResult& gz, Tensor norm_w, double eps,
                          Tensor state, Tensor seqs, int64_t S, Tensor o_raw, Tensor out) {
    CHECK_DT(qkv, at::kFloat); CHECK_DT(state, at::kFloat); CHECK_DT(out, at::kHalf);
    CHECK_DT(o_raw, at::kFloat); CHECK_DT(seqs, at::kInt); CHECK_CONTIG(qkv); CHECK_CONTIG(out);
    TORCH_CHECK(qkv.size(-1) == (2 * nk + nv) * D, "qkv width");
    TORCH_CHECK(o_raw.numel() >= out.numel(), "o_raw too small");
    const at::cuda::CUDAGuard guard(out.device());
    int rc = launch_delta_chunk(qkv.data_ptr<float>(), (int)qkv.size(-1), (int)nk, (int)nv, (int)D,
                                gba.g, dt_bias.data_ptr<float>(), A.data_ptr<float>(), gz.g,
                                norm_w.data_ptr<float>(), (float)eps, state.data_ptr<float>(),
                                seqs.data_ptr(), (int)S, (int)out.size(0), o_raw.data_ptr<float>(),
                                reinterpret_cast<__half*>(out.data_ptr()), cur_stream());
    TORCH_CHECK(rc == 0, "delta_chunk failed: rc=", rc);
  });
  m.def("delta_rule", [](Tensor qkv, int64_t nk, int64_t nv, int64_t D, const GemmResult& gba,
                         Tensor dt_bias, Tensor A, const GemmResult& gz, Tensor norm_w, double eps,
                         Tensor state, Tensor seqs, int64_t S, Tensor out) {
    CHECK_DT(qkv, at::kFloat); CHECK_DT(state, at::kFloat); CHECK_DT(out, at::kHalf);
    CHECK_DT(seqs, at::kInt); CHECK_CONTIG(qkv); CHECK_CONTIG(out);
    TORCH_CHECK(qkv.size(-1) == (2 * nk + nv) * D, "qkv width");
    const at::cuda::CUDAGuard guard(out.device());
    int rc = launch_delta_rule(qkv.data_ptr<float>(), (int)qkv.size(-1), (int)nk, (int)nv, (int)D,
                               gba.g, dt_bias.data_ptr<float>(), A.data_ptr<float>(), gz.g,
                               norm_w.data_ptr<float>(), (float)eps, state.data_ptr<float>(),
                               seqs.data_ptr(), (int)S, reinterpret_cast<__half*>(out.data_ptr()),
                               cur_stream());
    TORCH_CHECK(rc == 0, "delta_rule failed: rc=", rc);
  });
  m.def("epi_swiglu", &epi_swiglu);
  m.def("epi_copy", &epi_copy);
  m.def("qmatmul_simt", &qmatmul_simt);
  m.def("q4k_tc_plan", &q4k_tc_plan_py, py::arg("rows"), py::arg("K"), py::arg("T"),
        py::arg("num_sms"), py::arg("fmt") = 0);
  m.def("q4k_plan_max_ctas", [](int64_t T, int64_t num_sms, int64_t fmt) {
    return q4k_plan_max_ctas((int)T, (int)num_sms, (int)fmt); },
        py::arg("T"), py::arg("num_sms"), py::arg("fmt") = 0);
  m.def("q4k_gemv_max_t", []() { return q4k_gemv_max_t(); });
  m.def("q4k_gemv_occupancy", [](int64_t T, int64_t fmt) {
    return q4k_gemv_occupancy((int)T, (int)fmt); }, py::arg("T"), py::arg("fmt") = 0);
  m.def("qfmt_of_ggml", [](int64_t t) { return qfmt_of_ggml((int)t); });
  m.def("qfmt_row_bytes", [](int64_t f) { return qfmt_row_bytes((int)f); });
  m.def("qfmt_repack", &qfmt_repack);
  m.def("qgemm_q4k_tc", &qgemm_q4k_tc, py::arg("w_packed"), py::arg("rows"), py::arg("K"),
        py::arg("x"), py::arg("ws"), py::arg("status"), py::arg("num_sms"), py::arg("fmt") = 0,
        py::arg("w_b") = py::none(), py::arg("fmt_b") = -1, py::arg("split_tile") = 0);
  m.def("qgemm_q4k_tc_tp", &qgemm_q4k_tc_tp, py::arg("w_packed"), py::arg("rows"), py::arg("K"),
        py::arg("x"), py::arg("status"), py::arg("num_sms"), py::arg("recv_base"),
        py::arg("src_stride"), py::arg("dst_ptrs"), py::arg("sig_ctl"), py::arg("sig_bases"),
        py::arg("sig_flag_off"), py::arg("rank"), py::arg("owner_tiles"), py::arg("fmt") = 0);
  m.def("tp_reduce_norm", &tp_reduce_norm);
  m.def("tp_local_norm", &tp_local_norm);
  m.def("mma_probe_shapes", []() {
    std::vector<std::tuple<int, int, int>> v;
    for (int i = 0; i < mma_probe_shapes(); ++i) {
      int ts, mm, nn;
      mma_probe_shape(i, &ts, &mm, &nn);
      v.emplace_back(ts, mm, nn);
    }
    return v;
  });
  m.def("mma_probe", [](int64_t shape, int64_t iters, Tensor cycles, int64_t group, int64_t mode,
                        int64_t spin) {
    CHECK_DT(cycles, at::kLong);
    const at::cuda::CUDAGuard guard(cycles.device());
    TORCH_CHECK(launch_mma_probe((int)shape, (int)iters, (int)group, (int)mode, (int)spin,
                                 (int)cycles.numel(),
                                 reinterpret_cast<long long*>(cycles.data_ptr<int64_t>()),
                                 cur_stream()) == 0, "mma_probe launch failed");
  }, py::arg("shape"), py::arg("iters"), py::arg("cycles"), py::arg("group") = 0,
     py::arg("mode") = 1, py::arg("spin") = 0);
  // Bounded wait for `world` epoch flags (flags: device address of uint32[world]);
  // timeout_ns <= 0 uses the kernels' default deadline (1 s).
  m.def("flag_wait", [](int64_t flags, int64_t world, Tensor ctl, int64_t slot, Tensor status,
                        int64_t code, int64_t timeout_ns) {
    const at::cuda::CUDAGuard guard(ctl.device());
    TORCH_CHECK(launch_flag_wait(reinterpret_cast<const void*>(flags), (int)world,
                                 ctl.data_ptr<int>(), (int)slot, status.data_ptr<int>(), (int)code,
                                 cur_stream(), (long long)timeout_ns) == 0,
                "flag_wait launch failed");
  }, py::arg("flags"), py::arg("world"), py::arg("ctl"), py::arg("slot"), py::arg("status"),
     py::arg("code"), py::arg("timeout_ns") = 0);
  m.def("q4k_repack", &q4k_repack);
  m.def("dense_gemm_tc", &dense_gemm_tc);
  m.def("dense_tc_plan", &dense_tc_plan_py);
  m.def("qgemm_set_trace", &qgemm_set_trace_py);
  m.def("decode_attn", &decode_attn);
  m.def("attn_tc", &attn_tc);
  m.def("attn_set_trace", [](OptT buf) { attn_set_trace(ptr_or_null<void>(buf)); });
  m.def("argmax", &argmax);
  m.def("sample", &sample);
  m.def("philox_uniform", &philox_uniform);
  m.def("apply_penalties", &apply_penalties);
  register_moe_ops(m);
  register_ep_ops(m);
}
