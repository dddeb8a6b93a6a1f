// Discrete-event simulator of one serving cluster.
//
// Replays a frozen workload (study_workload rows) on `gpus` GPUs.  At every
// arrival or quantum completion it calls the same cluster_plan as the real
// executor, so the two share one planner; quantum durations come from the
// execution cost model, while the planner may be given a different
// `planner_cost` to model cost-model error.  Block preemption stops a rung
// video at its next doorbell check (estimate_preemption_timing).
// Reference: benchmarks/src/cluster_sim.cpp:27-354.
#pragma once
#include <string>

#include "ds/cost.hpp"
#include "ds/json.hpp"

namespace ds {

struct SimResult {
  Json rows;      // workload rows with status / finish_ms / start_ms
  Json summary;   // request_summary(rows)
  Json counters;  // plans, quanta, preemptions, resizes, batches
};

SimResult simulate_cluster(const Json& workload, int gpus, const std::string& policy, const ClusterCost& cost,
                           const Json& options = Json::object(), const ClusterCost* planner_cost = nullptr,
                           double horizon_ms = 1e12);

}  // namespace ds
