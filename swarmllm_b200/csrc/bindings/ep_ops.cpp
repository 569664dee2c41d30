// Torch bindings of the expert-parallel peer-memory kernels (ep_comm.cu).
#include "ops_common.h"

namespace {

py::tuple ep_arena_alloc_py(int64_t bytes) {
  void* p = nullptr;
  char h[64];
  const int rc = ep_arena_alloc((long long)bytes, &p, h);
  TORCH_CHECK(rc == 0, "ep arena allocation / IPC handle failed: rc=", rc);
  return py::make_tuple((int64_t)(uintptr_t)p, py::bytes(h, 64));
}

int64_t ep_arena_open_py(py::bytes handle) {
  std::string h = handle;
  TORCH_CHECK(h.size() == 64, "IPC handle must be 64 bytes");
  void* p = nullptr;
  TORCH_CHECK(ep_arena_open(h.data(), &p) == 0, "cudaIpcOpenMemHandle failed");
  return (int64_t)(uintptr_t)p;
}

// Non-owning tensor over [base + offset, ...) of an arena on `device`.
Tensor ep_view(int64_t base, int64_t offset, std::vector<int64_t> shape, std::string dtype,
               int64_t device) {
  at::ScalarType dt;
  if (dtype == "bf16") dt = at::kBFloat16;
  else if (dtype == "f16") dt = at::kHalf;
  else if (dtype == "f32") dt = at::kFloat;
  else if (dtype == "i32") dt = at::kInt;
  else TORCH_CHECK(false, "ep_view dtype must be bf16/f16/f32/i32");
  auto opts = at::TensorOptions().dtype(dt).device(at::kCUDA, (int)device);
  return torch::from_blob(reinterpret_cast<void*>(base + offset), shape, opts);
}

void ep_dispatch(Tensor x, Tensor ids, int64_t k, Tensor counts, int64_t E, int64_t e_loc,
                 int64_t cap, Tensor cursor, std::vector<int64_t> bases, int64_t rank,
                 bool x_bf16, Tensor ctl) {
  CHECK_DT(x, at::kHalf); CHECK_DT(ids, at::kInt); CHECK_DT(counts, at::kInt);
  CHECK_DT(cursor, at::kInt); CHECK_DT(ctl, at::kInt);
  TORCH_CHECK(x.stride(-1) == 1, "x rows must be contiguous");
  const at::cuda::CUDAGuard guard(x.device());
  unsigned long long b[8] = {0};
  for (size_t i = 0; i < bases.size() && i < 8; ++i) b[i] = (unsigned long long)bases[i];
  const int rc = launch_ep_dispatch(
      reinterpret_cast<const __half*>(x.data_ptr()), (int)x.stride(0), (int)x.size(1),
      ids.data_ptr<int32_t>(), (int)ids.numel(), (int)k, counts.data_ptr<int>(), (int)E,
      (int)e_loc, (int)cap, cursor.data_ptr<int>(), b, (int)bases.size(), (int)rank,
      x_bf16 ? 1 : 0, ctl.data_ptr<int>(), cur_stream());
  TORCH_CHECK(rc == 0, "ep_dispatch failed: rc=", rc);
}

void ep_wait(int64_t own_base, int64_t world, int64_t cap, int64_t H, int64_t e_loc,
             int64_t which, Tensor ctl, Tensor status, int64_t timeout_ns) {
  const at::cuda::CUDAGuard guard(ctl.device());
  TORCH_CHECK(launch_ep_wait((unsigned long long)own_base, (int)world, (int)cap, (int)H,
                             (int)e_loc, (int)which, ctl.data_ptr<int>(), status.data_ptr<int>(),
                             cur_stream(), (long long)timeout_ns) == 0, "ep_wait launch failed");
}

void ep_plan_owner(int64_t own_base, int64_t world, int64_t cap, int64_t H, int64_t e_loc,
                   int64_t tok_tile, Tensor tiles, Tensor n_tiles, Tensor status) {
  CHECK_DT(tiles, at::kInt); CHECK_DT(n_tiles, at::kInt);
  const at::cuda::CUDAGuard guard(tiles.device());
  TORCH_CHECK(launch_ep_plan_owner((unsigned long long)own_base, (int)world, (int)cap, (int)H,
                                   (int)e_loc, (int)tok_tile, tiles.data_ptr(),
                                   n_tiles.data_ptr<int>(), (int)tiles.size(0),
                                   status.data_ptr<int>(), cur_stream()) == 0,
              "ep_plan_owner launch failed");
}

py::tuple ep_arena_offsets_py(int64_t world, int64_t cap, int64_t H, int64_t e_loc) {
  long long o[6];
  ep_arena_offsets((int)world, (int)cap, (int)H, (int)e_loc, o);
  return py::make_tuple(o[0], o[1], o[2], o[3], o[4], o[5]);
}

}  // namespace

void register_ep_ops(py::module& m) {
  m.def("ep_arena_bytes", &ep_arena_bytes);
  m.def("ep_arena_offsets", &ep_arena_offsets_py);
  m.def("ep_arena_alloc", &ep_arena_alloc_py);
  m.def("ep_arena_open", &ep_arena_open_py);
  m.def("ep_arena_close", [](int64_t p, bool own) {
    return ep_arena_close(reinterpret_cast<void*>(p), own ? 1 : 0);
  });
  m.def("ep_view", &ep_view);
  m.def("ep_dispatch", &ep_dispatch);
  m.def("ep_wait", &ep_wait, py::arg("own_base"), py::arg("world"), py::arg("cap"), py::arg("H"),
        py::arg("e_loc"), py::arg("which"), py::arg("ctl"), py::arg("status"),
        py::arg("timeout_ns") = 0);
  m.def("ep_plan_owner", &ep_plan_owner);
}
