#include "ds/policy.hpp"

#include <map>
#include <mutex>
#include <set>
#include <stdexcept>

namespace ds {
namespace {

PolicyTraits base(const std::string& id, const std::string& display, const std::string& family,
                  const std::string& source) {
  PolicyTraits t;
  t.id = id;
  t.display = display;
  t.family = family;
  t.source = source;
  return t;
}

// the full system: block preemption, CFG-aware pruned forms, CFG-pair admission,
// pair-preserving image placement, continuous image batching with packing
PolicyTraits full(const std::string& id, const std::string& display, const std::string& family,
                  const std::string& source) {
  PolicyTraits t = base(id, display, family, source);
  t.elastic = t.blocks = t.prune_dominated = true;
  t.min_video_degree = 2;
  t.widen = 0.90;
  t.image_placement = "pair_fit";
  t.continuous_batch = t.sequence_packing = t.bubble_free = true;
  t.feasibility_guards = t.idle_widening = true;
  return t;
}

PolicyTraits knapsack_v1(const std::string& id, const std::string& display, const std::string& family,
                         const std::string& source) {
  PolicyTraits t = base(id, display, family, source);
  t.elastic = t.knapsack = true;
  t.widen = 0.90;
  t.image_placement = "pair_fit";
  return t;
}

std::map<std::string, PolicyTraits> build_table() {
  std::map<std::string, PolicyTraits> m;
  auto put = [&](PolicyTraits t) { m.emplace(t.id, std::move(t)); };
  put(full("ditserve", "DitServe", "ours", "block preemption, pruned CFG x SP forms, CFG-pair admission, continuous image batching"));
  {
    auto t = full("ditserve-b200", "DitServe (B200)", "ours",
                  "ditserve tuned on the measured B200 profile: load-adaptive forms (when the denoising videos "
                  "could fill every CFG pair, each video takes its most GPU-efficient form and feasibility is "
                  "judged on it; otherwise feasible-minimal forms with widening) and atomic images instead of "
                  "continuous image batches (images that are already late share continuous batches)");
    t.load_adaptive = true;
    t.continuous_batch = false;
    t.late_image_batching = true;
    put(t);
  }
  {
    auto t = full("ditserve-wide", "DitServe (widest form)", "diagnostic",
                  "ditserve whose videos start on their widest form while per-GPU efficiency stays >= 0.85 "
                  "(near-linear SP scaling over NVSwitch makes the wide form fastest at no extra GPU time)");
    t.wide_efficiency = 0.85;
    put(t);
  }
  {
    auto t = full("ditserve-approx", "DitServe-Approx", "ours", "ditserve plus late-step CFG folding (approximate)");
    t.v5 = t.fission = true;
    put(t);
  }
  {
    auto t = base("tetriserve", "TetriServe (re-impl.)", "baseline",
                  "round-based elastic SP sized by a deadline group knapsack; no sub-step preemption");
    t.elastic = t.rounds = t.deadline_dp = true;
    put(t);
  }
  {
    auto t = base("sbp-esp", "SBP-ESP", "baseline",
                  "step-boundary preemption, per-step deadline knapsack over videos, image batches up to 4");
    t.elastic = t.deadline_dp = t.image_batching = true;
    put(t);
  }
  {
    auto t = base("edf-bestfit", "EDF-BF", "baseline",
                  "strict EDF, smallest deadline-meeting group else largest fitting, surplus redistribution");
    t.elastic = t.best_fit = true;
    t.demote_late = false;
    put(t);
  }
  for (const char* id : {"tetriserve-cfg2", "sbp-esp-cfg2", "edf-bestfit-cfg2"}) {
    std::string parent(id);
    parent = parent.substr(0, parent.size() - 5);
    auto t = m.at(parent);
    t.id = id;
    t.display = t.display + "-CFG2";
    t.source = t.source + "; CFG=2 forms allowed";
    t.allow_cfg_forms = true;
    put(t);
  }
  {
    auto t = base("edf-cfg2", "EDF-CFG2", "heuristic", "every video on one CFG pair, EDF, images at step boundaries");
    t.fixed_form = parse_form("cfg2");
    t.fixed_degree = 2;
    put(t);
  }
  {
    auto t = base("cfg2-first", "CFG2-First", "heuristic",
                  "elastic over non-dominated forms, never narrower than a CFG pair, no sub-step preemption");
    t.elastic = t.prune_dominated = true;
    t.min_video_degree = 2;
    t.widen = 0.90;
    t.image_placement = "pair_fit";
    put(t);
  }
  {
    auto t = base("partition", "Static-Partition", "heuristic", "videos on fixed CFG pairs, a fixed image share");
    t.fixed_form = parse_form("cfg2");
    t.fixed_degree = 2;
    t.partition_divisor = 4;
    put(t);
  }
  auto ablate = [&](const char* id, const char* display, const char* what, auto edit) {
    auto t = full(id, display, "ablation", what);
    edit(t);
    put(t);
  };
  ablate("abl-no-block", "DitServe w/o block preemption", "whole-step quanta", [](PolicyTraits& t) { t.blocks = false; });
  ablate("abl-no-prune", "DitServe w/o form pruning", "no dominated-form pruning",
         [](PolicyTraits& t) { t.prune_dominated = false; });
  ablate("abl-no-mindeg", "DitServe w/o CFG-pair admission", "videos admitted on any group size",
         [](PolicyTraits& t) { t.min_video_degree = 1; });
  ablate("abl-first-fit", "DitServe w/o pair-fit placement", "images on the lowest free GPU",
         [](PolicyTraits& t) { t.image_placement = "first"; });
  ablate("abl-no-decode-shrink", "DitServe w/o decode shrink", "full video group held during decode",
         [](PolicyTraits& t) { t.hold_diffuse = true; });
  ablate("abl-no-img-priority", "DitServe w/o feasible image priority", "pure EDF between modalities",
         [](PolicyTraits& t) { t.feasible_img_priority = false; });
  ablate("abl-no-cb", "DitServe-noCB", "no continuous image batching, packing or bubble-free overlap",
         [](PolicyTraits& t) { t.continuous_batch = t.sequence_packing = t.bubble_free = false; });
  auto stair = [&](const char* id, const char* display, bool prune, int mindeg, double widen, const char* placement,
                   bool img_prio) {
    auto t = base(id, display, "ablation", "cumulative design staircase rung");
    t.elastic = true;
    t.prune_dominated = t.allow_cfg_forms = prune;
    t.min_video_degree = mindeg;
    t.widen = widen;
    t.image_placement = placement;
    t.feasible_img_priority = img_prio;
    put(t);
  };
  stair("stair-base", "Base (Step-SP)", false, 1, 0.0, "first", false);
  stair("stair-prune", "+Prune (CFG2 + L* Frontier)", true, 2, 0.0, "first", false);
  stair("stair-pairfit", "+PairFit (Online Scheduler)", true, 2, 0.90, "pair_fit", true);
  {
    auto t = knapsack_v1("ditserve-v1", "DitServe-v1 (knapsack)", "ablation", "earlier planner: block quanta + utility knapsack");
    t.blocks = t.tiered_memory = t.image_batching = true;
    put(t);
  }
  {
    auto t = knapsack_v1("ditserve-v1-approx", "DitServe-v1-Approx", "ablation", "utility knapsack + CFG folding");
    t.blocks = t.v5 = t.fission = true;
    put(t);
  }
  {
    auto t = base("abl-step-elastic", "Step-Elastic", "ablation", "elastic SP regrouped at every step boundary");
    t.elastic = true;
    put(t);
  }
  {
    auto t = base("abl-block-elastic", "Block-Elastic", "ablation", "step-elastic plus block quanta and lazy preemption");
    t.elastic = t.blocks = true;
    put(t);
  }
  {
    auto t = base("abl-round-elastic", "Round-Elastic", "ablation", "elastic SP regrouped every round_steps steps");
    t.elastic = t.rounds = true;
    put(t);
  }
  {
    auto t = knapsack_v1("diag-feature-cache", "Feature-Cache (diag.)", "diagnostic", "whole-step feature cache, SP1 pinned");
    t.approx = t.tiered_memory = t.image_batching = true;
    put(t);
  }
  {
    auto t = knapsack_v1("diag-v3", "HeteroDiT-v3 (diag.)", "diagnostic", "INT8 ring + Taylor + CFG reuse");
    t.approx = t.v3 = t.tiered_memory = t.image_batching = true;
    put(t);
  }
  {
    auto t = base("diag-tiered", "Tiered-State (diag.)", "diagnostic", "block-elastic with tiered host state");
    t.elastic = t.blocks = t.tiered_memory = true;
    put(t);
  }
  {
    auto t = base("diag-2d-usp", "2D-USP (diag.)", "diagnostic", "block-elastic over Ulysses x ring forms");
    t.elastic = t.blocks = t.tiered_memory = true;
    put(t);
  }
  {
    auto t = base("diag-elastic-partition", "Elastic-Partition (diag.)", "diagnostic", "step-elastic videos, reserved image GPUs");
    t.elastic = true;
    t.partition_divisor = 4;
    put(t);
  }
  return m;
}

const std::map<std::string, PolicyTraits>& table() {
  static const std::map<std::string, PolicyTraits> t = build_table();
  return t;
}

const std::map<std::string, std::string>& aliases() {
  static const std::map<std::string, std::string> a = {
      {"heterodit_exact", "ditserve-v1"}, {"knapsack_dp", "ditserve-v1"}, {"heterodit_v5", "ditserve-v1-approx"},
      {"step_elastic", "abl-step-elastic"}, {"block_elastic", "abl-block-elastic"},
      {"round_elastic", "abl-round-elastic"}, {"heterodit_approx", "diag-feature-cache"}, {"heterodit_v3", "diag-v3"},
      {"ablation_tiered", "diag-tiered"}, {"ablation_2d_usp", "diag-2d-usp"},
      {"static_partition", "diag-elastic-partition"}};
  return a;
}

const std::set<std::string>& retired() {
  static const std::set<std::string> r = {"vanilla_xdit", "tridentserve_stage", "vllm_omni", "gf_dit", "genserve_40gb"};
  return r;
}

bool split_parameterised(const std::string& name, std::string& kind, Form& form) {
  for (const char* prefix : {"static-", "block-", "xdit-", "fold-", "approx-", "static_", "block_"}) {
    const std::string p(prefix);
    if (name.compare(0, p.size(), p) != 0) continue;
    try {
      form = parse_form(name.substr(p.size()));
    } catch (const std::invalid_argument&) {
      throw std::invalid_argument("unknown cluster policy: " + name);
    }
    kind = p.substr(0, p.size() - 1);
    return true;
  }
  return false;
}

}  // namespace

std::string legacy_policy_alias(const std::string& name) {
  auto it = aliases().find(name);
  if (it != aliases().end()) return it->second;
  std::string kind;
  Form form;
  if (name.find('_') != std::string::npos && name.find('-') == std::string::npos &&
      split_parameterised(name, kind, form))
    return kind + "-" + form_name(form);
  return "";
}

std::string canonical_policy(const std::string& name) {
  if (name == "xdit") return "xdit-sp1";
  std::string legacy = legacy_policy_alias(name);
  return legacy.empty() ? name : legacy;
}

const PolicyTraits& policy_traits(const std::string& raw) {
  if (retired().count(raw)) throw std::invalid_argument("retired cluster policy: " + raw);
  const std::string name = canonical_policy(raw);
  auto it = table().find(name);
  if (it != table().end()) return it->second;
  std::string kind;
  Form form;
  if (!split_parameterised(name, kind, form)) throw std::invalid_argument("unknown cluster policy: " + raw);
  static std::mutex mu;
  static std::map<std::string, PolicyTraits> cache;
  std::lock_guard<std::mutex> lock(mu);
  auto c = cache.find(name);
  if (c != cache.end()) return c->second;
  const std::string fname = form_name(form);
  PolicyTraits t;
  if (kind == "static") {
    t = base(name, "Static-" + fname, "control", "fixed parallel form, EDF, whole-step quanta");
  } else if (kind == "block") {
    t = base(name, "Block-" + fname, "control", "fixed parallel form with block quanta and sub-step preemption");
    t.blocks = true;
  } else if (kind == "fold" || kind == "approx") {
    t = base(name, (kind == "fold" ? "Fold-" : "Approx-") + fname, "ablation",
             kind == "fold" ? "fixed-form CFG folding, unconditional subgroup idle" : "fixed CFG form with folding and fission");
    t.blocks = t.v5 = true;
    t.fission = kind == "approx";
  } else {
    t = base(name, fname == "sp1" ? "xDiT" : "xDiT-" + fname, "baseline",
             "xDiT static partition: fixed form per video, image share gpus/4, FCFS, run to completion");
    t.hold_diffuse = true;
    t.order = "fcfs";
    t.demote_late = false;
    t.partition_divisor = 4;
  }
  t.fixed_form = form;
  t.fixed_degree = form.degree();
  return cache.emplace(name, t).first->second;
}

Json describe_policy(const PolicyTraits& t) {
  Json j = Json::object();
  j["id"] = t.id;
  j["display"] = t.display;
  j["family"] = t.family;
  j["source"] = t.source;
  j["fixed_form"] = t.fixed_degree ? form_name(t.fixed_form) : std::string();
  j["elastic"] = t.elastic;
  j["blocks"] = t.blocks;
  j["rounds"] = t.rounds;
  j["knapsack"] = t.knapsack;
  j["deadline_dp"] = t.deadline_dp;
  j["best_fit"] = t.best_fit;
  j["approximate"] = t.approx || t.v3 || t.v5;
  j["fission"] = t.fission;
  j["prune_dominated"] = t.prune_dominated;
  j["min_video_degree"] = t.min_video_degree;
  j["order"] = t.order;
  j["hold_diffuse"] = t.hold_diffuse;
  j["partition_divisor"] = t.partition_divisor;
  j["demote_late"] = t.demote_late;
  j["widen"] = t.widen;
  j["wide_efficiency"] = t.wide_efficiency;
  j["load_adaptive"] = t.load_adaptive;
  j["image_placement"] = t.image_placement;
  j["image_batching"] = t.image_batching;
  j["round_steps"] = t.round_steps;
  j["allow_cfg_forms"] = t.allow_cfg_forms;
  j["feasible_img_priority"] = t.feasible_img_priority;
  j["continuous_batch"] = t.continuous_batch;
  j["sequence_packing"] = t.sequence_packing;
  j["bubble_free"] = t.bubble_free;
  j["feasibility_guards"] = t.feasibility_guards;
  j["idle_widening"] = t.idle_widening;
  j["late_image_batching"] = t.late_image_batching;
  return j;
}

Json policy_catalog() {
  Json out = Json::array();
  for (const auto& kv : table()) out.push_back(describe_policy(kv.second));
  for (const char* n : {"xdit-sp1", "xdit-sp2", "xdit-cfg2", "static-cfg2", "block-cfg2", "fold-cfg2sp3", "approx-cfg2sp3"})
    out.push_back(describe_policy(policy_traits(n)));
  return out;
}

}  // namespace ds
