#include "planner.h"

#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <algorithm>
#include <limits>

namespace py = pybind11;

namespace swarm_native {

StagePlan plan_bottleneck(const std::vector<double>& layer_cost,
                          const std::vector<double>& layer_mem,
                          const std::vector<double>& dev_speed,
                          const std::vector<double>& dev_mem, double hop_cost) {
  const int L = (int)layer_cost.size(), S = (int)dev_speed.size();
  StagePlan plan;
  if (L == 0 || S == 0 || S > L) return plan;
  std::vector<double> pc(L + 1, 0.0), pm(L + 1, 0.0);
  for (int l = 0; l < L; ++l) {
    pc[l + 1] = pc[l] + layer_cost[l];
    pm[l + 1] = pm[l] + (layer_mem.empty() ? 0.0 : layer_mem[l]);
  }
  const double INF = std::numeric_limits<double>::infinity();
  // best[s][l]: minimal bottleneck placing layers [0, l) on stages [0, s).
  std::vector<std::vector<double>> best(S + 1, std::vector<double>(L + 1, INF));
  std::vector<std::vector<double>> sum(S + 1, std::vector<double>(L + 1, INF));
  std::vector<std::vector<int>> arg(S + 1, std::vector<int>(L + 1, -1));
  best[0][0] = 0.0;
  sum[0][0] = 0.0;
  for (int s = 1; s <= S; ++s) {
    const double speed = dev_speed[s - 1] > 0 ? dev_speed[s - 1] : 1.0;
    for (int l = s; l <= L - (S - s); ++l) {
      for (int k = s - 1; k < l; ++k) {
        if (best[s - 1][k] == INF) continue;
        if (!dev_mem.empty() && pm[l] - pm[k] > dev_mem[s - 1]) continue;
        const double c = (pc[l] - pc[k]) / speed + (s > 1 ? hop_cost : 0.0);
        const double b = std::max(best[s - 1][k], c);
        const double t = sum[s - 1][k] + c;
        if (b < best[s][l] || (b == best[s][l] && t < sum[s][l])) {
          best[s][l] = b;
          sum[s][l] = t;
          arg[s][l] = k;
        }
      }
    }
  }
  if (best[S][L] == INF) return plan;
  plan.feasible = true;
  plan.bottleneck = best[S][L];
  plan.total = sum[S][L];
  plan.first_layer.assign(S + 1, 0);
  int l = L;
  for (int s = S; s >= 1; --s) {
    plan.first_layer[s] = l;
    l = arg[s][l];
  }
  plan.first_layer[0] = 0;
  return plan;
}

StagePlan plan_route(const std::vector<double>& layer_cost, const std::vector<double>& layer_mem,
                     const std::vector<double>& dev_speed, const std::vector<double>& dev_mem,
                     const std::vector<double>& dev_load, double hop_cost,
                     std::vector<int>* devices_out) {
  // Shortest path over states (layer boundary l, last device d): a device may
  // be used once, in index order (devices are interchangeable on NVSwitch; the
  // order fixes one canonical route).
  const int L = (int)layer_cost.size(), D = (int)dev_speed.size();
  StagePlan plan;
  if (L == 0 || D == 0) return plan;
  std::vector<double> pc(L + 1, 0.0), pm(L + 1, 0.0);
  for (int l = 0; l < L; ++l) {
    pc[l + 1] = pc[l] + layer_cost[l];
    pm[l + 1] = pm[l] + (layer_mem.empty() ? 0.0 : layer_mem[l]);
  }
  const double INF = std::numeric_limits<double>::infinity();
  // dist[d][l]: best latency covering [0, l) with the last stage on device d.
  std::vector<std::vector<double>> dist(D, std::vector<double>(L + 1, INF));
  std::vector<std::vector<std::pair<int, int>>> prev(D, std::vector<std::pair<int, int>>(L + 1, {-1, -1}));
  for (int d = 0; d < D; ++d) {
    const double load = dev_load.empty() ? 1.0 : std::max(1.0, dev_load[d]);
    const double speed = (dev_speed[d] > 0 ? dev_speed[d] : 1.0) / load;
    for (int l = 1; l <= L; ++l) {
      // first stage from layer 0
      if (dev_mem.empty() || pm[l] <= dev_mem[d]) {
        const double c = pc[l] / speed;
        if (c < dist[d][l]) { dist[d][l] = c; prev[d][l] = {-1, 0}; }
      }
      for (int pd = 0; pd < d; ++pd) {
        for (int k = 1; k < l; ++k) {
          if (dist[pd][k] == INF) continue;
          if (!dev_mem.empty() && pm[l] - pm[k] > dev_mem[d]) continue;
          const double c = dist[pd][k] + hop_cost + (pc[l] - pc[k]) / speed;
          if (c < dist[d][l]) { dist[d][l] = c; prev[d][l] = {pd, k}; }
        }
      }
    }
  }
  int bd = -1;
  double bv = INF;
  for (int d = 0; d < D; ++d)
    if (dist[d][L] < bv) { bv = dist[d][L]; bd = d; }
  if (bd < 0) return plan;
  std::vector<int> devs, bounds;
  int d = bd, l = L;
  while (d >= 0) {
    devs.push_back(d);
    bounds.push_back(l);
    auto [pd, k] = prev[d][l];
    l = k;
    d = pd;
  }
  bounds.push_back(0);
  std::reverse(devs.begin(), devs.end());
  std::reverse(bounds.begin(), bounds.end());
  plan.feasible = true;
  plan.total = bv;
  plan.first_layer = bounds;
  double bn = 0;
  for (size_t i = 0; i < devs.size(); ++i) {
    const double load = dev_load.empty() ? 1.0 : std::max(1.0, dev_load[devs[i]]);
    bn = std::max(bn, (pc[bounds[i + 1]] - pc[bounds[i]]) * load / dev_speed[devs[i]]);
  }
  plan.bottleneck = bn;
  if (devices_out) *devices_out = devs;
  return plan;
}

void bind_planner(py::module_& m) {
  py::class_<StagePlan>(m, "StagePlan")
      .def_readonly("first_layer", &StagePlan::first_layer)
      .def_readonly("bottleneck", &StagePlan::bottleneck)
      .def_readonly("total", &StagePlan::total)
      .def_readonly("feasible", &StagePlan::feasible);
  m.def("plan_bottleneck", &plan_bottleneck, py::arg("layer_cost"), py::arg("layer_mem"),
        py::arg("dev_speed"), py::arg("dev_mem"), py::arg("hop_cost") = 0.0);
  m.def(
      "plan_route",
      [](const std::vector<double>& lc, const std::vector<double>& lm,
         const std::vector<double>& sp, const std::vector<double>& mem,
         const std::vector<double>& load, double hop) {
        std::vector<int> devs;
        StagePlan p = plan_route(lc, lm, sp, mem, load, hop, &devs);
        return py::make_tuple(p, devs);
      },
      py::arg("layer_cost"), py::arg("layer_mem"), py::arg("dev_speed"), py::arg("dev_mem"),
      py::arg("dev_load"), py::arg("hop_cost") = 0.0);
}

}  // namespace swarm_native
