// Layer-range planner: cut a model's layers into contiguous stages.
//
// The reference plans each request's chain of peers with a shortest-path DP
// over layer ranges, priced by measured per-layer latency, RTT and load
// (route_shortest_path, src/inference/scheduler/parallax.rs:1154;
// chain_cost_terms at :1040).  On one NVSwitch box every link costs the same,
// so two objectives matter and both are solved exactly by DP over
// (stage, first layer):
//   * throughput: minimise the slowest stage (pipeline bottleneck) subject to
//     each stage's memory capacity;
//   * latency: minimise the sum of stage times + per-hop link cost over a
//     chosen subset of devices (a request's route).
#pragma once
#include <cstdint>
#include <vector>

namespace pybind11 {
class module_;
}

namespace swarm_native {

struct StagePlan {
  std::vector<int> first_layer;  // [S+1] boundaries, stage s = [b[s], b[s+1])
  double bottleneck = 0.0;       // max stage cost
  double total = 0.0;            // sum of stage costs + hop costs
  bool feasible = false;
};

// layer_cost[l]: time of layer l on a unit-speed device; layer_mem[l]: bytes.
// dev_speed[s], dev_mem[s]: speed factor (time divides by it) and capacity.
StagePlan plan_bottleneck(const std::vector<double>& layer_cost,
                          const std::vector<double>& layer_mem,
                          const std::vector<double>& dev_speed,
                          const std::vector<double>& dev_mem, double hop_cost);

// Choose, in order, a subset of the devices and a layer range for each to
// minimise end-to-end latency (sum of stage times + hop cost per boundary).
// Returns (device index per used stage, boundaries).
StagePlan plan_route(const std::vector<double>& layer_cost, const std::vector<double>& layer_mem,
                     const std::vector<double>& dev_speed, const std::vector<double>& dev_mem,
                     const std::vector<double>& dev_load, double hop_cost,
                     std::vector<int>* devices_out);

void bind_planner(pybind11::module_& m);

}  // namespace swarm_native
