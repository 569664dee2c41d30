#include "tree.h"

#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <algorithm>
#include <stdexcept>

namespace py = pybind11;

namespace swarm_native {

DraftTree::DraftTree(int32_t root_token, int max_nodes) : max_nodes_(std::min(max_nodes, 64)) {
  TreeNode r;
  r.token = root_token;
  r.mask = 1ull;
  nodes_.push_back(r);
  frontier_.push_back(0);
}

std::vector<int32_t> DraftTree::expand(const std::vector<int32_t>& cand_tok,
                                       const std::vector<float>& cand_logp, int k, int width) {
  struct Cand {
    double logp;
    int32_t parent, token;
  };
  std::vector<Cand> cands;
  if (cand_tok.size() != frontier_.size() * (size_t)k || cand_logp.size() != cand_tok.size())
    throw std::invalid_argument("expand: candidates must be frontier.size() * k");
  for (size_t i = 0; i < frontier_.size(); ++i) {
    const int p = frontier_[i];
    for (int j = 0; j < k; ++j)
      cands.push_back({nodes_[p].logp + cand_logp[i * k + j], p, cand_tok[i * k + j]});
  }
  std::stable_sort(cands.begin(), cands.end(), [](const Cand& a, const Cand& b) { return a.logp > b.logp; });
  std::vector<int32_t> nf;
  for (const Cand& c : cands) {
    if ((int)nf.size() >= width || (int)nodes_.size() >= max_nodes_) break;
    // skip duplicate siblings
    bool dup = false;
    for (int32_t n : nf)
      if (nodes_[n].parent == c.parent && nodes_[n].token == c.token) { dup = true; break; }
    if (dup) continue;
    TreeNode n;
    n.token = c.token;
    n.parent = c.parent;
    n.depth = nodes_[c.parent].depth + 1;
    n.logp = c.logp;
    n.mask = nodes_[c.parent].mask | (1ull << nodes_.size());
    nf.push_back((int32_t)nodes_.size());
    nodes_.push_back(n);
  }
  frontier_ = nf;
  return nf;
}

std::pair<std::vector<int32_t>, int32_t> DraftTree::walk(const std::vector<int32_t>& target) const {
  if (target.size() < nodes_.size()) throw std::invalid_argument("walk: need a target token per node");
  std::vector<int32_t> path{0};
  int cur = 0;
  while (true) {
    const int32_t want = target[cur];
    int next = -1;
    for (size_t i = 1; i < nodes_.size(); ++i)
      if (nodes_[i].parent == cur && nodes_[i].token == want) { next = (int)i; break; }
    if (next < 0) return {path, want};
    path.push_back(next);
    cur = next;
  }
}

std::vector<int32_t> DraftTree::tokens() const {
  std::vector<int32_t> v;
  for (auto& n : nodes_) v.push_back(n.token);
  return v;
}
std::vector<int32_t> DraftTree::depths() const {
  std::vector<int32_t> v;
  for (auto& n : nodes_) v.push_back(n.depth);
  return v;
}
std::vector<int32_t> DraftTree::parents() const {
  std::vector<int32_t> v;
  for (auto& n : nodes_) v.push_back(n.parent);
  return v;
}
std::vector<uint64_t> DraftTree::masks() const {
  std::vector<uint64_t> v;
  for (auto& n : nodes_) v.push_back(n.mask);
  return v;
}

void bind_tree(py::module_& m) {
  py::class_<DraftTree>(m, "DraftTree")
      .def(py::init<int32_t, int>(), py::arg("root_token"), py::arg("max_nodes") = 64)
      .def("__len__", &DraftTree::size)
      .def("frontier", &DraftTree::frontier)
      .def("expand", &DraftTree::expand, py::arg("cand_tok"), py::arg("cand_logp"), py::arg("k"),
           py::arg("width"))
      .def("walk", &DraftTree::walk)
      .def("tokens", &DraftTree::tokens)
      .def("depths", &DraftTree::depths)
      .def("parents", &DraftTree::parents)
      .def("masks", &DraftTree::masks);
}

}  // namespace swarm_native
