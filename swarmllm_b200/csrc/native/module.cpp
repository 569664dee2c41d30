// pybind11 module swarmllm_b200._native: the C++ runtime pieces.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "block_manager.h"
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

  bind_gguf(m);
  bind_planner(m);
  bind_tree(m);
}
