// Cluster planner shared by the real executor and the simulator.
//
// cluster_plan(state, policy, cost, options) decides, at one instant, which
// waiting or suspended requests start a quantum on which GPUs.
//
// state:   {now_ms, gpus, busy: [bool], async_decoding?: [bool], requests: [...], sp_groups_running}
//          (a GPU with an asynchronous VAE decode in flight takes images but no new video)
// request: {request_id, kind video|image, class, arrival_ms, deadline_ms,
//           status waiting|suspended, steps_done, blocks_done, steps_total?,
//           group [] (last GPUs held), form (last form), decode_done, affinity?}
// options: forms / degrees (candidate video forms), order, widen_efficiency,
//          image_placement, min_video_degree, prune_dominated, demote_late,
//          partition_image_gpus, round_steps, quantum_blocks, continuous_batch
//          (max members), image_batch, sequence_packing, pairing, ...
//          (each overrides the policy's default trait).
// returns: {assignments: [{request_id, group, degree, form, quantum, steps?,
//           resize, reason, batch?, pair?, decode_frames?}], preempt: [ids],
//           deadline_skips}
//
// GPUs are interchangeable on NVSwitch, so "aligned" groups only keep a
// request's ranks contiguous (cheap resharding, readable traces); the planner
// never pays a placement penalty.  Behaviours per policy come from
// PolicyTraits (policy.hpp); reference planner: src/ditserve/control/cluster.cpp:788-2283.
#pragma once
#include <string>
#include <vector>

#include "ds/cost.hpp"
#include "ds/json.hpp"
#include "ds/policy.hpp"

namespace ds {

std::vector<std::vector<int>> cluster_groups(int gpus, int size);

// bounded, decision-free diagnostic sink
struct PlanTrace {
  size_t max_rows = 64;
  Json rows = Json::array();
  size_t dropped = 0;
  void add(const Json& row);
};

Json cluster_plan(const Json& state, const std::string& policy, const ClusterCost& cost,
                  const Json& options = Json::object(), PlanTrace* trace = nullptr);

// forms a policy may use for `klass` on `gpus` GPUs (after pruning)
std::vector<Form> candidate_forms(const PolicyTraits& t, const ClusterCost& cost, const std::string& klass, int gpus,
                                  const Json& options);

// ---- block preemption (sub-step, through doorbells) ------------------------
struct PreemptionTiming {
  double stop_ms = 0, remaining_ms = 0;
};
// block_ms per rank-local block; the flag is polled every check_blocks blocks
// (blocks_per_iteration per poll when branches interleave); a delayed group
// check (the poll consumes the previous checkpoint's flag) doubles the stop time.
PreemptionTiming estimate_preemption_timing(double block_ms, int blocks_total, int blocks_done, double elapsed_ms,
                                            int check_blocks, int blocks_per_iteration, bool delayed_group_check);
// true when stopping early turns this image from late into on time
bool preemption_converts_deadline(double now_ms, double deadline_ms, double service_ms, double stop_ms,
                                  double boundary_ms);

struct RunningGroup {
  std::string request_id;
  std::vector<int> group;
  double stop_ms = 0, remaining_ms = 0, resume_ms = 0;
  bool rung = false;
};
struct ImageDemand {
  int affinity = -1;  // -1: any GPU
  double deadline_ms = 0, service_ms = 0;
};
// min-cost selection of running groups to free enough GPUs for the waiting images
std::vector<std::string> select_preemption_groups(const std::vector<int>& image_affinities,
                                                  const std::vector<RunningGroup>& running);
struct DeadlinePreemption {
  std::vector<std::string> selected;
  size_t deadline_skips = 0;
};
// EDF demand matching: each newly rung group must save the image it is matched to
DeadlinePreemption select_deadline_preemption(double now_ms, const std::vector<ImageDemand>& waiting,
                                              const std::vector<RunningGroup>& running);

}  // namespace ds
