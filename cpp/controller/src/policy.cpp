#include "ds/policy.hpp"

#include <map>
#include <mutex>
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

// ---------------------------------------------------------------------------
// Name resolution
//
// Three kinds of name besides the registered ids:
//  * exact names from older studies: either an alias (it resolves to another name) or a
//    retired policy (resolving it is an error that says so);
//  * "xdit" on its own, the single-GPU xDiT baseline;
//  * family names "<kind>-<form>" (a fixed parallel form, see form.hpp).  Two families were
//    also written "<kind>_<form>" in older studies; that spelling is accepted only in a
//    name without any '-', and it canonicalises to the '-' spelling.
// A name that claims a family kind but carries a malformed form is an error, never a
// silent fallback to another policy.

enum class OldName { kAlias, kRetired };
struct OldNameRule {
  const char* name;
  OldName what;
  const char* target;  // alias target (unused for retired names)
};
constexpr OldNameRule kOldNames[] = {
    {"heterodit_exact", OldName::kAlias, "ditserve-v1"},
    {"knapsack_dp", OldName::kAlias, "ditserve-v1"},
    {"heterodit_v5", OldName::kAlias, "ditserve-v1-approx"},
    {"step_elastic", OldName::kAlias, "abl-step-elastic"},
    {"block_elastic", OldName::kAlias, "abl-block-elastic"},
    {"round_elastic", OldName::kAlias, "abl-round-elastic"},
    {"heterodit_approx", OldName::kAlias, "diag-feature-cache"},
    {"heterodit_v3", OldName::kAlias, "diag-v3"},
    {"ablation_tiered", OldName::kAlias, "diag-tiered"},
    {"ablation_2d_usp", OldName::kAlias, "diag-2d-usp"},
    {"static_partition", OldName::kAlias, "diag-elastic-partition"},
    {"vanilla_xdit", OldName::kRetired, ""},
    {"tridentserve_stage", OldName::kRetired, ""},
    {"vllm_omni", OldName::kRetired, ""},
    {"gf_dit", OldName::kRetired, ""},
    {"genserve_40gb", OldName::kRetired, ""},
};

const OldNameRule* old_name(const std::string& name) {
  for (const auto& r : kOldNames)
    if (name == r.name) return &r;
  return nullptr;
}

// What a family name implies.  Every family runs one fixed form chosen by the name.
struct FamilySpec {
  const char* kind;
  bool underscore_spelling;  // also accepted as "<kind>_<form>" (older studies)
  const char* family;
  const char* display;       // display prefix; the form name follows
  const char* source;
  bool blocks, v5, fission;
  bool xdit_partition;       // the xDiT static partition: FCFS, run to completion, a quarter of the GPUs for images
  bool cfg_only;             // only meaningful with CFG parallelism (listed with cfg2 forms in the catalog)
};
constexpr FamilySpec kFamilies[] = {
    {"static", true, "control", "Static-", "fixed parallel form, EDF, whole-step quanta", false, false, false, false,
     false},
    {"block", true, "control", "Block-", "fixed parallel form with block quanta and sub-step preemption", true, false,
     false, false, false},
    {"fold", false, "ablation", "Fold-", "fixed-form CFG folding, unconditional subgroup idle", true, true, false,
     false, true},
    {"approx", false, "ablation", "Approx-", "fixed CFG form with folding and fission", true, true, true, false, true},
    {"xdit", false, "baseline", "xDiT-",
     "xDiT static partition: fixed form per video, image share gpus/4, FCFS, run to completion", false, false, false,
     true, false},
};

const FamilySpec* family_of(const std::string& kind) {
  for (const auto& f : kFamilies)
    if (kind == f.kind) return &f;
  return nullptr;
}

struct FamilyName {
  const FamilySpec* spec = nullptr;
  char separator = '-';
  Form form;
};

// Splits "<kind><sep><form>" at the first separator.  Returns false when the name does not
// claim a family (no separator, an unknown kind, or '_' for a family without that spelling);
// throws when it claims one and the form part is malformed.
bool read_family_name(const std::string& name, FamilyName& out) {
  const size_t cut = name.find_first_of("-_");
  if (cut == std::string::npos) return false;
  const FamilySpec* spec = family_of(name.substr(0, cut));
  if (spec == nullptr) return false;
  if (name[cut] == '_' && !spec->underscore_spelling) return false;
  try {
    out.form = parse_form(name.substr(cut + 1));
  } catch (const std::invalid_argument&) {
    throw std::invalid_argument("unknown cluster policy: " + name);
  }
  out.spec = spec;
  out.separator = name[cut];
  return true;
}

PolicyTraits family_traits(const std::string& id, const FamilyName& fn) {
  const FamilySpec& f = *fn.spec;
  const std::string form = form_name(fn.form);
  const std::string display =
      f.xdit_partition && form == "sp1" ? std::string("xDiT") : std::string(f.display) + form;
  PolicyTraits t = base(id, display, f.family, f.source);
  t.blocks = f.blocks;
  t.v5 = f.v5;
  t.fission = f.fission;
  if (f.xdit_partition) {
    t.hold_diffuse = true;
    t.order = "fcfs";
    t.demote_late = false;
    t.partition_divisor = 4;
  }
  t.fixed_form = fn.form;
  t.fixed_degree = fn.form.degree();
  return t;
}

// Traits of family names are built on first use and kept for the life of the process, so
// the references handed out stay valid.
class FamilyRegistry {
 public:
  const PolicyTraits& get(const std::string& id, const FamilyName& fn) {
    std::lock_guard<std::mutex> lock(mu_);
    auto it = built_.find(id);
    if (it == built_.end()) it = built_.emplace(id, family_traits(id, fn)).first;
    return it->second;
  }

 private:
  std::mutex mu_;
  std::map<std::string, PolicyTraits> built_;
};

FamilyRegistry& families() {
  static FamilyRegistry r;
  return r;
}

}  // namespace

std::string legacy_policy_alias(const std::string& name) {
  if (const OldNameRule* r = old_name(name)) return r->what == OldName::kAlias ? r->target : "";
  FamilyName fn;
  const bool old_spelling = name.find('-') == std::string::npos && name.find('_') != std::string::npos;
  if (old_spelling && read_family_name(name, fn) && fn.separator == '_')
    return std::string(fn.spec->kind) + "-" + form_name(fn.form);
  return "";
}

std::string canonical_policy(const std::string& name) {
  if (name == "xdit") return "xdit-sp1";
  const std::string alias = legacy_policy_alias(name);
  return alias.empty() ? name : alias;
}

const PolicyTraits& policy_traits(const std::string& raw) {
  if (const OldNameRule* r = old_name(raw); r != nullptr && r->what == OldName::kRetired)
    throw std::invalid_argument("retired cluster policy: " + raw);
  const std::string id = canonical_policy(raw);
  const auto& registered = table();
  if (auto it = registered.find(id); it != registered.end()) return it->second;
  FamilyName fn;
  if (!read_family_name(id, fn)) throw std::invalid_argument("unknown cluster policy: " + raw);
  return families().get(id, fn);
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
  // registered ids, then every family on the fixed forms of this framework's default layouts
  // for 1, 2, 4 and 8 GPUs (sp1, cfg2, cfg2sp2, cfg2sp4); families that need CFG parallelism
  // are listed on the cfg2 forms only
  Json out = Json::array();
  for (const auto& kv : table()) out.push_back(describe_policy(kv.second));
  for (const auto& f : kFamilies)
    for (const char* form : {"sp1", "cfg2", "cfg2sp2", "cfg2sp4"}) {
      if (f.cfg_only && parse_form(form).cfg != 2) continue;
      out.push_back(describe_policy(policy_traits(std::string(f.kind) + "-" + form)));
    }
  return out;
}

}  // namespace ds
