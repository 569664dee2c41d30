// pybind11 module swarmllm_b200._native: the C++ runtime pieces.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <optional>

#include "block_manager.h"
#include "cpu_attn.h"
#include "cpu_qmatmul.h"
#include "gguf_reader.h"
#include "planner.h"
#include "scheduler.h"
#include "tree.h"

namespace py = pybind11;
using namespace swarm_native;

template <typename T>
static py::array_t<T> to_np(const std::vector<T>& v) {
  py::array_t<T> a(v.size());
  if (!v.empty()) std::copy(v.begin(), v.end(), a.mutable_data());
  return a;
}

PYBIND11_MODULE(_native, m) {
  m.doc() = "swarmllm_b200 native runtime (block manager, scheduler, GGUF, planners)";

  py::class_<BlockManager>(m, "BlockManager")
      .def(py::init<int, int, bool>(), py::arg("num_pages"), py::arg("page_size"),
           py::arg("prefix_cache") = true)
      .def_property_readonly("page_size", &BlockManager::page_size)
      .def_property_readonly("num_pages", &BlockManager::num_pages)
      .def("num_free", &BlockManager::num_free)
      .def("add_sequence", &BlockManager::add_sequence, py::arg("seq_id"), py::arg("tokens"),
           py::arg("salt") = 0, py::arg("cap") = -1, py::arg("exact") = false)
      .def("chain_hashes", &BlockManager::chain_hashes, py::arg("tokens"), py::arg("n_pages"),
           py::arg("salt") = 0)
      .def("has_sequence", &BlockManager::has_sequence)
      .def("seq_len", &BlockManager::seq_len)
      .def("append_slots", [](BlockManager& b, int64_t id, int n) { return to_np(b.append_slots(id, n)); })
      .def("can_append", &BlockManager::can_append)
      .def("commit_tokens", &BlockManager::commit_tokens)
      .def("truncate", &BlockManager::truncate)
      .def("fork", &BlockManager::fork)
      .def("free_sequence", &BlockManager::free_sequence)
      .def("pages", [](const BlockManager& b, int64_t id) { return to_np(b.pages(id)); })
      .def("block_table",
           [](const BlockManager& b, const std::vector<int64_t>& ids, int max_pages) {
             py::array_t<int32_t> a({(py::ssize_t)ids.size(), (py::ssize_t)max_pages});
             b.fill_block_table(ids, max_pages, a.mutable_data());
             return a;
           })
      .def("cached_prefix_pages",
           [](const BlockManager& b, const std::vector<int32_t>& t, uint64_t salt) {
             return to_np(b.cached_prefix_pages(t, salt));
           }, py::arg("tokens"), py::arg("salt") = 0)
      .def("import_prefix_pages",
           [](BlockManager& b, const std::vector<int32_t>& t, int n, uint64_t salt) {
             return to_np(b.import_prefix_pages(t, n, salt));
           }, py::arg("tokens"), py::arg("n_pages"), py::arg("salt") = 0)
      .def_property_readonly("prefix_hit_tokens", &BlockManager::prefix_hits)
      .def_property_readonly("num_cached_pages", &BlockManager::num_cached_pages);

  py::class_<StepPlan>(m, "StepPlan")
      .def_property_readonly("seq_ids", [](const StepPlan& p) { return to_np(p.seq_ids); })
      .def_property_readonly("seq_start", [](const StepPlan& p) { return to_np(p.seq_start); })
      .def_property_readonly("seq_ntok", [](const StepPlan& p) { return to_np(p.seq_ntok); })
      .def_property_readonly("seq_sample", [](const StepPlan& p) { return to_np(p.seq_sample); })
      .def_property_readonly("tokens", [](const StepPlan& p) { return to_np(p.tokens); })
      .def_property_readonly("positions", [](const StepPlan& p) { return to_np(p.positions); })
      .def_property_readonly("slots", [](const StepPlan& p) { return to_np(p.slots); })
      .def_property_readonly("row_seq", [](const StepPlan& p) { return to_np(p.row_seq); })
      .def_readonly("n_decode", &StepPlan::n_decode)
      .def_readonly("n_prefill_tokens", &StepPlan::n_prefill_tokens)
      .def("__len__", [](const StepPlan& p) { return p.tokens.size(); });

  py::class_<Scheduler>(m, "Scheduler")
      .def(py::init<BlockManager*, int, int, int>(), py::arg("block_manager"),
           py::arg("max_step_tokens"), py::arg("max_running"), py::arg("prefill_chunk"),
           py::keep_alive<1, 2>())
      .def("add_request", &Scheduler::add_request, py::arg("id"), py::arg("prompt"),
           py::arg("max_new"), py::arg("eos") = -1, py::arg("cache_salt") = 0,
           py::arg("max_cover") = -1, py::arg("cover_exact") = false, py::arg("split_at") = -1)
      .def("abort", &Scheduler::abort)
      .def("schedule", &Scheduler::schedule)
      .def("commit", &Scheduler::commit)
      .def("output", [](const Scheduler& s, int64_t id) { return to_np(s.request(id).output); })
      .def("finished", [](const Scheduler& s, int64_t id) { return s.request(id).finished; })
      .def("release", &Scheduler::release)
      .def_property_readonly("num_waiting", &Scheduler::num_waiting)
      .def_property_readonly("num_running", &Scheduler::num_running)
      .def_property_readonly("num_preemptions", &Scheduler::num_preemptions)
      .def("has_work", &Scheduler::has_work);

  m.def(
      "cpu_qmatmul",
      [](py::array_t<uint8_t, py::array::c_style> w, int type, int rows, int K,
         py::array_t<float, py::array::c_style | py::array::forcecast> x) {
        if (x.ndim() != 2 || x.shape(1) != K) throw std::invalid_argument("x must be [T, K]");
        const int T = (int)x.shape(0);
        py::array_t<float> out({(py::ssize_t)T, (py::ssize_t)rows});
        const uint8_t* wp = w.data();
        const float* xp = x.data();
        float* op = out.mutable_data();
        int rc;
        {
          py::gil_scoped_release nogil;
          rc = cpu_qmatmul(wp, type, rows, K, xp, T, op);
        }
        if (rc != 0) throw std::invalid_argument("cpu_qmatmul: unsupported type or K");
        return out;
      },
      py::arg("w"), py::arg("type"), py::arg("rows"), py::arg("K"), py::arg("x"),
      "x [T, K] fp32 times the GGUF-quantized W [rows, K]^T, int8 activations, OpenMP rows");
  m.def("cpu_qmatmul_isa", [] { return std::string(cpu_qmatmul_isa()); });
  m.def(
      "cpu_dequant",
      [](py::array_t<uint8_t, py::array::c_style> w, int type, int rows, int K) {
        py::array_t<float> out({(py::ssize_t)rows, (py::ssize_t)K});
        const uint8_t* wp = w.data();
        float* op = out.mutable_data();
        int rc;
        {
          py::gil_scoped_release nogil;
          rc = cpu_dequant(wp, type, rows, K, op);
        }
        if (rc != 0) throw std::invalid_argument("cpu_dequant: unsupported type or K");
        return out;
      },
      py::arg("w"), py::arg("type"), py::arg("rows"), py::arg("K"),
      "the fp32 values of `rows` rows of GGUF blocks");

  using f32a = py::array_t<float, py::array::c_style | py::array::forcecast>;
  using i32a = py::array_t<int32_t, py::array::c_style | py::array::forcecast>;
  m.def(
      "cpu_paged_attention",
      [](f32a q, py::array k_cache, py::array v_cache, i32a block_table, i32a seq_lens,
         float scale, int window, float softcap, std::optional<i32a> tree_start,
         std::optional<py::array_t<int64_t, py::array::c_style | py::array::forcecast>> tree_mask,
         std::optional<f32a> sinks) {
        if (q.ndim() != 3 || k_cache.ndim() != 4 || v_cache.ndim() != 4 || block_table.ndim() != 2)
          throw std::invalid_argument("q [N,H,d], caches [pages,kv,ps,d], block_table [N,P]");
        const bool f16 = k_cache.dtype().is(py::dtype("float16"));
        if (!f16 && !k_cache.dtype().is(py::dtype::of<float>()))
          throw std::invalid_argument("KV cache must be float16 or float32");
        if (!k_cache.dtype().is(v_cache.dtype()))
          throw std::invalid_argument("K and V caches differ in dtype");
        if (!(k_cache.flags() & py::array::c_style) || !(v_cache.flags() & py::array::c_style))
          throw std::invalid_argument("KV caches must be contiguous");
        AttnArgs a{};
        a.n_tokens = (int)q.shape(0);
        a.n_heads = (int)q.shape(1);
        a.head_dim = (int)q.shape(2);
        a.n_kv_heads = (int)k_cache.shape(1);
        a.page_size = (int)k_cache.shape(2);
        a.max_pages = (int)block_table.shape(1);
        if (k_cache.shape(3) != a.head_dim || block_table.shape(0) != a.n_tokens ||
            seq_lens.size() != a.n_tokens)
          throw std::invalid_argument("shape mismatch");
        py::array_t<float> out({q.shape(0), q.shape(1), q.shape(2)});
        a.q = q.data();
        a.out = out.mutable_data();
        a.block_table = block_table.data();
        a.seq_lens = seq_lens.data();
        a.tree_start = tree_start ? tree_start->data() : nullptr;
        a.tree_mask = tree_mask ? tree_mask->data() : nullptr;
        a.sinks = sinks ? sinks->data() : nullptr;
        a.window = window;
        a.scale = scale;
        a.softcap = softcap;
        const void* kp = k_cache.data();
        const void* vp = v_cache.data();
        int rc;
        {
          py::gil_scoped_release nogil;
          rc = cpu_paged_attention(a, kp, vp, f16);
        }
        if (rc != 0) throw std::invalid_argument("cpu_paged_attention: bad head counts");
        return out;
      },
      py::arg("q"), py::arg("k_cache"), py::arg("v_cache"), py::arg("block_table"),
      py::arg("seq_lens"), py::arg("scale"), py::arg("window") = 0, py::arg("softcap") = 0.f,
      py::arg("tree_start") = py::none(), py::arg("tree_mask") = py::none(),
      py::arg("sinks") = py::none(),
      "paged attention of q [N, H, d] over fp16/fp32 caches [pages, kv, page, d]");
  m.def(
      "cpu_silu_mul",
      [](f32a g, f32a u, float limit, float alpha) {
        if (g.size() != u.size()) throw std::invalid_argument("g and u differ in size");
        py::array_t<float> out(std::vector<py::ssize_t>(g.shape(), g.shape() + g.ndim()));
        const float* gp = g.data();
        const float* up = u.data();
        float* op = out.mutable_data();
        const int64_t n = g.size();
        {
          py::gil_scoped_release nogil;
          cpu_silu_mul(gp, up, op, n, limit, alpha);
        }
        return out;
      },
      py::arg("g"), py::arg("u"), py::arg("limit") = 0.f, py::arg("alpha") = 1.702f);
  m.def(
      "cpu_delta_rule",
      [](f32a q, f32a k, f32a v, f32a g, f32a beta,
         py::array_t<float, py::array::c_style> state) {
        if (q.ndim() != 3 || k.ndim() != 3 || v.ndim() != 3 || state.ndim() != 3)
          throw std::invalid_argument("q, k [T, nk, dk], v [T, nv, dv], state [nv, dk, dv]");
        const int T = (int)q.shape(0), nk = (int)q.shape(1), dk = (int)q.shape(2);
        const int nv = (int)v.shape(1), dv = (int)v.shape(2);
        if (k.shape(0) != T || k.shape(1) != nk || k.shape(2) != dk || v.shape(0) != T ||
            g.size() != (py::ssize_t)T * nv || beta.size() != (py::ssize_t)T * nv ||
            state.shape(0) != nv || state.shape(1) != dk || state.shape(2) != dv ||
            nk <= 0 || nv % nk != 0)
          throw std::invalid_argument("delta rule shapes");
        if (!state.writeable()) throw std::invalid_argument("state must be writeable");
        py::array_t<float> out({(py::ssize_t)T, (py::ssize_t)nv, (py::ssize_t)dv});
        const float *qp = q.data(), *kp = k.data(), *vp = v.data(), *gp = g.data(),
                    *bp = beta.data();
        float* sp = state.mutable_data();
        float* op = out.mutable_data();
        {
          py::gil_scoped_release nogil;
          cpu_delta_rule(qp, kp, vp, gp, bp, sp, op, T, nk, nv, dk, dv);
        }
        return out;
      },
      py::arg("q"), py::arg("k"), py::arg("v"), py::arg("g"), py::arg("beta"), py::arg("state"),
      "gated delta rule over T rows; state [nv, dk, dv] fp32 updated in place");
  m.def("exp_approx", [](f32a x) {
    py::array_t<float> out(std::vector<py::ssize_t>(x.shape(), x.shape() + x.ndim()));
    for (py::ssize_t i = 0; i < x.size(); ++i) out.mutable_data()[i] = exp_approx(x.data()[i]);
    return out;
  });

  bind_gguf(m);
  bind_planner(m);
  bind_tree(m);
}
