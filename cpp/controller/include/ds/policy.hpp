// Scheduling-policy registry.  One PolicyTraits record per policy id holds
// every behaviour the name implies, so the planner, the executor and the
// simulator consult facts instead of comparing names.  The ids, families and
// trait values are the reference registry's (src/ditserve/control/policy.cpp:36-265)
// so study configurations and result records stay interchangeable; the
// descriptions are ours.  Parameterised names: static-<form>, block-<form>,
// xdit-<form>, fold-<form>, approx-<form>.
#pragma once
#include <string>

#include "ds/form.hpp"
#include "ds/json.hpp"

namespace ds {

struct PolicyTraits {
  std::string id, display, family, source;
  Form fixed_form;
  int fixed_degree = 0;           // 0: planner chooses the form
  bool elastic = false;           // regroup at step boundaries
  bool blocks = false;            // block quanta + sub-step (doorbell) preemption
  bool rounds = false;            // regroup only every round_steps steps
  bool knapsack = false;          // v1 utility knapsack
  bool deadline_dp = false;       // 0/1 deadline group knapsack (requests kept on track)
  bool best_fit = false;          // EDF best fit + surplus redistribution
  bool approx = false, v3 = false, v5 = false, fission = false;
  double widen = 0.0;             // widen a video when per-GPU efficiency stays >= widen
  bool widen_past_images = false;  // widening continues while images wait (they preempt by doorbell)
  double feasible_margin = 0.0;    // slack kept by the feasible-minimal form choice (fraction of remaining)
  double wide_efficiency = 0.0;    // >0: videos start on their widest form whose per-GPU efficiency stays above it
  bool load_adaptive = false;      // many videos: the most GPU-efficient form; few: the usual choice
  std::string image_placement = "first";  // first | pair_fit
  bool hold_diffuse = false;      // a started video keeps its GPUs (no decode shrink)
  bool demote_late = true;        // late requests ranked behind feasible ones
  std::string order = "edf";      // edf | srtf | fcfs
  bool prune_dominated = false;   // drop forms that a no-wider form beats
  int min_video_degree = 1;
  int partition_divisor = 0;      // >0: gpus / divisor GPUs reserved for images
  int round_steps = 5;
  bool tiered_memory = false;
  bool image_batching = false;
  bool pin_started = false;
  bool allow_cfg_forms = false;
  bool feasible_img_priority = true;
  bool continuous_batch = false;
  bool sequence_packing = false;
  bool bubble_free = false;
  // feasibility guards of the full system: a video does not widen to meet its own deadline
  // when that leaves two or more feasible videos without GPUs; an in-flight video past half
  // of its steps with a small overrun keeps its rank (sunk-work deadband); a step-boundary
  // video does not migrate to another group of the same size when the resize would make it
  // late; images take GPUs that the highest-laxity suspended video holds
  bool feasibility_guards = false;
  bool idle_widening = false;     // widen below the efficiency threshold onto GPUs nobody else needs
  bool late_image_batching = false;  // late images share continuous batches though on-time ones run alone
};

const PolicyTraits& policy_traits(const std::string& name);  // throws std::invalid_argument
std::string canonical_policy(const std::string& name);
std::string legacy_policy_alias(const std::string& name);     // "" when not an alias
Json policy_catalog();
Json describe_policy(const PolicyTraits& t);

}  // namespace ds
