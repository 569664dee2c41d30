// Torch bindings of the mixture-of-experts kernels (moe_tc.cu).
#include "ops_common.h"

namespace {

void moe_topk(const GemmResult& lg, OptT br, int64_t T, int64_t E, int64_t k, int64_t mode,
              OptT sel_b, bool norm, double scale, Tensor ids, Tensor wts, Tensor counts) {
  CHECK_DT(ids, at::kInt); CHECK_DT(wts, at::kFloat); CHECK_DT(counts, at::kInt);
  TORCH_CHECK(lg.g.rows == E && lg.g.T >= T, "router logits shape");
  TORCH_CHECK(ids.numel() >= T * k && wts.numel() >= T * k, "ids/wts too small");
  if (sel_b.has_value()) {
    CHECK_DT((*sel_b), at::kFloat);
    TORCH_CHECK(sel_b->numel() >= E, "selection bias too small");
  }
  const at::cuda::CUDAGuard guard(ids.device());
  int rc = launch_moe_topk(lg.g, ptr_or_null<float>(br), (int)T, (int)E, (int)k, (int)mode,
                           ptr_or_null<float>(sel_b), norm ? 1 : 0, (float)scale,
                           ids.data_ptr<int32_t>(), wts.data_ptr<float>(),
                           counts.data_ptr<int>(), cur_stream());
  TORCH_CHECK(rc == 0, "moe_topk failed: rc=", rc);
}

void moe_plan(Tensor counts, int64_t E, int64_t tok_tile, Tensor offsets, Tensor cursor,
              Tensor tiles, Tensor n_tiles, Tensor status) {
  CHECK_DT(counts, at::kInt); CHECK_DT(offsets, at::kInt); CHECK_DT(cursor, at::kInt);
  CHECK_DT(tiles, at::kInt); CHECK_DT(n_tiles, at::kInt);
  TORCH_CHECK(tiles.dim() == 2 && tiles.size(1) == 4, "tiles must be [max_tiles, 4]");
  TORCH_CHECK(offsets.numel() >= E + 1, "offsets must hold E+1");
  const at::cuda::CUDAGuard guard(counts.device());
  int rc = launch_moe_plan(counts.data_ptr<int>(), (int)E, (int)tok_tile, offsets.data_ptr<int>(),
                           cursor.data_ptr<int>(), tiles.data_ptr(), n_tiles.data_ptr<int>(),
                           (int)tiles.size(0), status.data_ptr<int>(), cur_stream());
  TORCH_CHECK(rc == 0, "moe_plan failed: rc=", rc);
}

void moe_scatter(Tensor x, Tensor ids, int64_t k, Tensor cursor, Tensor xs, Tensor ret,
                 int64_t rank) {
  CHECK_DT(x, at::kHalf); CHECK_DT(ids, at::kInt); CHECK_DT(ret, at::kInt);
  TORCH_CHECK(xs.scalar_type() == at::kHalf || xs.scalar_type() == at::kBFloat16, "xs dtype");
  TORCH_CHECK(x.stride(-1) == 1 && xs.stride(-1) == 1, "rows must be contiguous");
  const at::cuda::CUDAGuard guard(x.device());
  const int P = (int)ids.numel();
  TORCH_CHECK(xs.size(0) >= P && ret.numel() >= P, "xs/ret too small");
  int rc = launch_moe_scatter(reinterpret_cast<const __half*>(x.data_ptr()), (int)x.stride(0),
                              (int)x.size(1), ids.data_ptr<int32_t>(), P, (int)k,
                              cursor.data_ptr<int>(), xs.data_ptr(), (int)xs.stride(0),
                              xs.scalar_type() == at::kBFloat16 ? 1 : 0, ret.data_ptr<int32_t>(),
                              (int)rank, cur_stream());
  TORCH_CHECK(rc == 0, "moe_scatter failed: rc=", rc);
}

void moe_gemm(int64_t fmt, int64_t epi, Tensor w, int64_t rows, int64_t K, Tensor xs,
              int64_t tok_tile, Tensor tiles, Tensor n_tiles, OptT bias, int64_t bias_stride,
              OptT h, int64_t act_kind, double alpha, double limit, std::vector<int64_t> out_ptrs,
              int64_t out_stride, OptT ret, int64_t num_sms, Tensor status, OptT sig_ctl,
              std::vector<int64_t> sig_bases, int64_t sig_flag_off, int64_t sig_rank) {
  CHECK_CUDA(w); CHECK_CUDA(xs); CHECK_DT(tiles, at::kInt); CHECK_DT(status, at::kInt);
  TORCH_CHECK(status.numel() >= 8, "status must hold 8 ints");
  TORCH_CHECK(xs.scalar_type() == (fmt == 1 ? at::kBFloat16 : at::kHalf),
              "xs must be bf16 for MXFP4 experts, fp16 for Q4_K experts");
  if (epi == 0) {
    TORCH_CHECK(h.has_value() && h->scalar_type() == xs.scalar_type(), "h dtype");
  } else {
    TORCH_CHECK(ret.has_value() && !out_ptrs.empty() && out_ptrs.size() <= 8, "store targets");
  }
  const at::cuda::CUDAGuard guard(xs.device());
  unsigned long long ptrs[8] = {0};
  for (size_t i = 0; i < out_ptrs.size() && i < 8; ++i) ptrs[i] = (unsigned long long)out_ptrs[i];
  TORCH_CHECK(sig_bases.size() <= 8, "at most 8 ranks");
  unsigned long long sb[8] = {0};
  for (size_t i = 0; i < sig_bases.size(); ++i) sb[i] = (unsigned long long)sig_bases[i];
  int rc = launch_moe_gemm_tc(
      (int)fmt, (int)epi, w.data_ptr(), (int)rows, (int)K, xs.data_ptr(), (int)xs.stride(0),
      (int)xs.size(0), (int)tok_tile, tiles.data_ptr(), n_tiles.data_ptr<int>(),
      (int)tiles.size(0), ptr_or_null<float>(bias), (int)bias_stride, ptr_or_null<void>(h),
      h.has_value() ? (int)h->stride(0) : 0, (int)act_kind, (float)alpha, (float)limit, ptrs,
      (int)out_ptrs.size(), (int)out_stride, ptr_or_null<int32_t>(ret),
      num_sms > 0 ? (int)num_sms : num_sms_of(xs), status.data_ptr<int>(), cur_stream(),
      ptr_or_null<int>(sig_ctl), sb, (long long)sig_flag_off, (int)sig_bases.size(),
      (int)sig_rank);
  TORCH_CHECK(rc == 0, "moe_gemm failed: rc=", rc);
}

void moe_combine(Tensor rows, Tensor wts, int64_t k, const GemmResult* sh, const GemmResult* shg,
                 Tensor residual, OptT norm_w, OptT out, double eps) {
  CHECK_DT(rows, at::kFloat); CHECK_DT(wts, at::kFloat); CHECK_DT(residual, at::kFloat);
  const at::cuda::CUDAGuard guard(residual.device());
  const int T = (int)residual.size(0), H = (int)residual.size(1);
  if (out.has_value()) CHECK_DT(*out, at::kHalf);
  int rc = launch_moe_combine(rows.data_ptr<float>(), (int)rows.stride(0), wts.data_ptr<float>(),
                              (int)k, sh ? &sh->g : nullptr, shg ? &shg->g : nullptr,
                              residual.data_ptr<float>(), T, H, ptr_or_null<float>(norm_w),
                              ptr_or_null<__half>(out), out.has_value() ? (int)out->stride(0) : 0,
                              (float)eps, cur_stream());
  TORCH_CHECK(rc == 0, "moe_combine failed: rc=", rc);
}

void moe_localize(Tensor ids, Tensor wts, Tensor counts, int64_t E, int64_t e0, int64_t n_loc) {
  CHECK_DT(ids, at::kInt); CHECK_DT(wts, at::kFloat); CHECK_DT(counts, at::kInt);
  const at::cuda::CUDAGuard guard(ids.device());
  TORCH_CHECK(launch_moe_localize(ids.data_ptr<int32_t>(), wts.data_ptr<float>(),
                                  counts.data_ptr<int>(), (int)ids.numel(), (int)E, (int)e0,
                                  (int)n_loc, cur_stream()) == 0, "moe_localize failed");
}

// This rank's MoE partial into the owners' receive slots; returns the dense
// GemmOut over all W slots of this rank's receive buffer (for tp_reduce_norm).
GemmResult moe_combine_tp(Tensor rows, Tensor wts, int64_t k, const GemmResult* sh,
                          const GemmResult* shg, int64_t T, int64_t H, int64_t recv_base,
                          int64_t src_stride, std::vector<int64_t> dst_ptrs, Tensor sig_ctl,
                          std::vector<int64_t> sig_bases, int64_t sig_flag_off, int64_t rank,
                          bool to_all) {
  CHECK_DT(rows, at::kFloat); CHECK_DT(wts, at::kFloat); CHECK_DT(sig_ctl, at::kInt);
  TORCH_CHECK(!dst_ptrs.empty() && dst_ptrs.size() <= 8 && dst_ptrs.size() == sig_bases.size(),
              "1..8 ranks");
  const at::cuda::CUDAGuard guard(rows.device());
  unsigned long long d[8], b[8];
  for (size_t i = 0; i < dst_ptrs.size(); ++i) {
    d[i] = (unsigned long long)dst_ptrs[i];
    b[i] = (unsigned long long)sig_bases[i];
  }
  const int W = (int)dst_ptrs.size();
  int rc = launch_moe_combine_tp(rows.data_ptr<float>(), (int)rows.stride(0), wts.data_ptr<float>(),
                                 (int)k, sh ? &sh->g : nullptr, shg ? &shg->g : nullptr, (int)T,
                                 (int)H, W, d, sig_ctl.data_ptr<int>(), b,
                                 (long long)sig_flag_off, (int)rank, cur_stream(), to_all ? 1 : 0);
  TORCH_CHECK(rc == 0, "moe_combine_tp failed: rc=", rc);
  GemmResult r;
  r.g = swarm::GemmOut{};
  r.g.ws = reinterpret_cast<const float*>(recv_base);
  r.g.rows = (int)H;
  r.g.T = (int)T;
  r.g.mode = 0;
  r.g.n_src = W;
  r.g.src_stride = src_stride;
  return r;
}

void mxfp4_repack(Tensor src, int64_t rows, int64_t K, Tensor dst) {
  CHECK_CUDA(src); CHECK_CUDA(dst);
  TORCH_CHECK(dst.numel() * dst.element_size() >= moe_packed_bytes(1, (int)rows, (int)K),
              "dst too small");
  const at::cuda::CUDAGuard guard(dst.device());
  TORCH_CHECK(launch_mxfp4_repack(src.data_ptr(), (int)rows, (int)K, dst.data_ptr(),
                                  cur_stream()) == 0, "mxfp4_repack failed");
}

}  // namespace

void register_moe_ops(py::module& m) {
  m.def("moe_topk", &moe_topk);
  m.def("moe_plan", &moe_plan);
  m.def("moe_scatter", &moe_scatter);
  m.def("moe_gemm", &moe_gemm, py::arg("fmt"), py::arg("epi"), py::arg("w"), py::arg("rows"),
        py::arg("K"), py::arg("xs"), py::arg("tok_tile"), py::arg("tiles"), py::arg("n_tiles"),
        py::arg("bias"), py::arg("bias_stride"), py::arg("h"), py::arg("act_kind"),
        py::arg("alpha"), py::arg("limit"), py::arg("out_ptrs"), py::arg("out_stride"),
        py::arg("ret"), py::arg("num_sms"), py::arg("status"), py::arg("sig_ctl") = py::none(),
        py::arg("sig_bases") = std::vector<int64_t>{}, py::arg("sig_flag_off") = 0,
        py::arg("sig_rank") = 0);
  m.def("moe_combine", &moe_combine, py::arg("rows"), py::arg("wts"), py::arg("k"),
        py::arg("sh").none(true), py::arg("shg").none(true), py::arg("residual"),
        py::arg("norm_w"), py::arg("out"), py::arg("eps"));
  m.def("moe_localize", &moe_localize);
  m.def("moe_combine_tp", &moe_combine_tp, py::arg("rows"), py::arg("wts"), py::arg("k"),
        py::arg("sh").none(true), py::arg("shg").none(true), py::arg("T"), py::arg("H"),
        py::arg("recv_base"), py::arg("src_stride"), py::arg("dst_ptrs"), py::arg("sig_ctl"),
        py::arg("sig_bases"), py::arg("sig_flag_off"), py::arg("rank"), py::arg("to_all") = false);
  m.def("mxfp4_repack", &mxfp4_repack);
  m.def("moe_packed_bytes", &moe_packed_bytes);
  m.def("moe_tok_tile", &moe_tok_tile);
  m.def("moe_max_tiles", &moe_max_tiles);
}
