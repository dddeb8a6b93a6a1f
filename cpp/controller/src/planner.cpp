#include "ds/planner.hpp"

#include <algorithm>
#include <cmath>
#include <limits>
#include <map>
#include <set>
#include <stdexcept>
#include <tuple>

namespace ds {

std::vector<std::vector<int>> cluster_groups(int gpus, int size) {
  std::vector<std::vector<int>> out;
  if (size <= 0) return out;
  for (int s = 0; s + size <= gpus; s += size) {
    std::vector<int> g;
    for (int i = 0; i < size; ++i) g.push_back(s + i);
    out.push_back(g);
  }
  return out;
}

void PlanTrace::add(const Json& row) {
  if (rows.size() < max_rows) rows.push_back(row);
  else ++dropped;
}

namespace {

constexpr double kInf = std::numeric_limits<double>::infinity();

struct Settings {
  PolicyTraits t;
  std::vector<int> degrees{1, 2, 4, 8};
  std::vector<Form> forms;  // explicit options.forms
  int quantum_blocks = 0;   // 0: whole step
  int continuous_batch = 0; // max members of a continuous image batch (0/1: off)
  int image_batch = 1;
  bool pairing = false;
  bool preempt = true;
  bool ring_forms = false;
  int partition_image_gpus = -1;
  int check_blocks = 1;
  bool widen_past_images = false;  // widen even while images wait (they preempt by doorbell)
  double feasible_margin = 0.0;     // feasible-min keeps this fraction of the remaining time as slack
  double wide_efficiency = 0.0;     // >0: videos start on their widest form at least this efficient
  double late_short_ms = 0.0;       // late requests this short keep their EDF position
  bool load_adaptive = false;       // many videos: most GPU-efficient form; few: normal choice
  double quantum_ms = 0.0;          // >0: block quanta sized to this much GPU time
  bool lazy_preemption = true;      // an image that can wait for a mid-step video's boundary does
  std::string feasibility_degree;   // "free" | "widest": the degree the lateness test assumes
  bool late_image_batching = false; // late images go to continuous batches even without the trait
};

Settings resolve(const PolicyTraits& t, const Json& o) {
  Settings s;
  s.t = t;
  if (o.contains("degrees")) {
    s.degrees.clear();
    for (const auto& d : o.at("degrees").as_array()) s.degrees.push_back(static_cast<int>(d.as_int()));
  }
  if (o.contains("forms"))
    for (const auto& f : o.at("forms").as_array()) s.forms.push_back(parse_form(f.as_string()));
  s.t.order = o.str("order", t.order);
  if (s.t.order != "edf" && s.t.order != "srtf" && s.t.order != "fcfs") throw std::invalid_argument("order must be edf, srtf or fcfs");
  s.t.widen = o.num("widen_efficiency", t.widen);
  s.t.image_placement = o.str("image_placement", t.image_placement);
  if (s.t.image_placement != "first" && s.t.image_placement != "pair_fit")
    throw std::invalid_argument("image_placement must be first or pair_fit");
  s.t.min_video_degree = static_cast<int>(o.integer("min_video_degree", t.min_video_degree));
  s.t.prune_dominated = o.flag("prune_dominated", t.prune_dominated);
  s.t.demote_late = o.flag("demote_late", t.demote_late);
  s.t.hold_diffuse = o.flag("hold_diffuse", t.hold_diffuse);
  s.t.round_steps = static_cast<int>(o.integer("round_steps", t.round_steps));
  s.t.allow_cfg_forms = o.flag("allow_cfg_forms", t.allow_cfg_forms);
  s.t.feasible_img_priority = o.flag("feasible_img_priority", t.feasible_img_priority);
  s.t.blocks = o.flag("block_preemption", t.blocks);
  s.t.sequence_packing = o.flag("sequence_packing", t.sequence_packing);
  s.t.bubble_free = t.continuous_batch && o.flag("bubble_free", t.bubble_free);
  s.quantum_blocks = static_cast<int>(o.integer("quantum_blocks", 0));
  // continuous batching is a capability of the policy: the phase option sizes it for the
  // policies that own it and the others ignore it, so options shared by every arm of a study
  // do not hand it to the baselines
  const int cb_option = static_cast<int>(o.integer("continuous_batch", 8));
  if (cb_option < 0 || cb_option > 8) throw std::invalid_argument("continuous_batch must be 0..8");
  s.continuous_batch = t.continuous_batch ? cb_option : 0;
  s.t.feasibility_guards = o.flag("feasibility_guards", t.feasibility_guards);
  s.t.idle_widening = o.flag("idle_widening", t.idle_widening);
  s.image_batch = static_cast<int>(o.integer("image_batch", t.image_batching ? 4 : 1));
  s.pairing = o.flag("pairing", false);
  s.preempt = o.flag("doorbell", true);
  s.ring_forms = o.flag("ring_forms", t.id == "diag-2d-usp");
  s.partition_image_gpus = static_cast<int>(o.integer("partition_image_gpus", -1));
  s.check_blocks = static_cast<int>(o.integer("check_blocks", 1));
  s.widen_past_images = o.flag("widen_past_images", t.widen_past_images);
  s.feasible_margin = o.num("feasible_margin", t.feasible_margin);
  s.wide_efficiency = o.num("wide_efficiency", t.wide_efficiency);
  s.late_short_ms = o.num("late_short_ms", 0.0);
  s.load_adaptive = o.flag("load_adaptive", t.load_adaptive);
  if (s.late_short_ms < 0) throw std::invalid_argument("late_short_ms must be >= 0");
  s.quantum_ms = o.num("quantum_ms", 0.0);
  if (!(s.quantum_ms >= 0)) throw std::invalid_argument("quantum_ms must be >= 0");
  s.lazy_preemption = o.flag("lazy_preemption", true);
  s.late_image_batching = o.flag("late_image_batching", t.late_image_batching);
  // elastic policies judge lateness on the widest group free when the plan starts (a request
  // that only an idle node could save would otherwise keep its rank, run narrow and miss);
  // static policies on their widest degree
  s.feasibility_degree = o.str("feasibility_degree", t.elastic ? "free" : "widest");
  if (s.feasibility_degree != "free" && s.feasibility_degree != "widest")
    throw std::invalid_argument("feasibility_degree must be free or widest");
  if (s.feasible_margin < 0 || s.feasible_margin > 10) throw std::invalid_argument("feasible_margin must be in [0, 10]");
  return s;
}

std::vector<Form> forms_for(const Settings& s, const ClusterCost& cost, const std::string& klass, int gpus) {
  const PolicyTraits& t = s.t;
  std::vector<Form> forms;
  if (t.fixed_degree > 0) {
    if (t.fixed_form.degree() <= gpus) forms.push_back(t.fixed_form);
    return forms;
  }
  const bool cfg_forms = t.allow_cfg_forms || t.prune_dominated || t.min_video_degree >= 2;
  if (!s.forms.empty()) {
    for (const auto& f : s.forms)
      if (f.degree() <= gpus && (cfg_forms || f.cfg == 1)) forms.push_back(f);
  } else {
    forms = enumerate_forms(s.degrees, cfg_forms, s.ring_forms, gpus);
  }
  const int heads = cost.heads(klass);
  if (heads > 0)
    forms.erase(std::remove_if(forms.begin(), forms.end(), [&](const Form& f) { return heads % f.ulysses() != 0; }),
                forms.end());
  if (t.prune_dominated && forms.size() > 1) {
    std::vector<Form> kept;
    for (const auto& f : forms) {
      const double sf = cost.step_ms(klass, f);
      bool dominated = false;
      for (const auto& g : forms) {
        if (g == f || g.degree() > f.degree()) continue;
        const double sg = cost.step_ms(klass, g);
        if (sg < sf || (sg == sf && g.degree() < f.degree())) {
          dominated = true;
          break;
        }
      }
      if (!dominated) kept.push_back(f);
    }
    if (!kept.empty()) forms = kept;
  }
  // classes whose weights or activations do not fit one GPU name a minimum degree
  const int class_min = cost.has_class(klass) ? static_cast<int>(cost.klass(klass).integer("min_degree", 1)) : 1;
  if (class_min > 1)
    forms.erase(std::remove_if(forms.begin(), forms.end(), [&](const Form& f) { return f.degree() < class_min; }),
                forms.end());
  // on hardware where SP scales near-linearly (NVLink/NVSwitch), a video runs fastest and
  // costs no more GPU time on its widest efficient form: start it there (serialising
  // videos) instead of sharing the node between narrow groups
  if (s.wide_efficiency > 0 && forms.size() > 1) {
    const Form* base = &forms.front();
    for (const auto& f : forms)
      if (f.degree() < base->degree()) base = &f;
    const double base_work = cost.step_ms(klass, *base) * base->degree();
    int widest = 0;
    for (const auto& f : forms)
      if (base_work / (cost.step_ms(klass, f) * f.degree()) >= s.wide_efficiency) widest = std::max(widest, f.degree());
    if (widest > 1)
      forms.erase(std::remove_if(forms.begin(), forms.end(), [&](const Form& f) { return f.degree() < widest; }),
                  forms.end());
  }
  if (t.min_video_degree > 1) {
    std::vector<Form> wide;
    for (const auto& f : forms)
      if (f.degree() >= t.min_video_degree) wide.push_back(f);
    if (!wide.empty()) forms = wide;
  }
  std::sort(forms.begin(), forms.end(), [&](const Form& a, const Form& b) {
    if (a.degree() != b.degree()) return a.degree() < b.degree();
    return cost.step_ms(klass, a) < cost.step_ms(klass, b);
  });
  // one form per degree: the fastest of that size
  std::vector<Form> best;
  for (const auto& f : forms)
    if (best.empty() || best.back().degree() != f.degree()) best.push_back(f);
  return best;
}

struct Req {
  const Json* j = nullptr;
  std::string id, kind, klass, status;
  double arrival = 0, deadline = 0;
  std::vector<int> group;
  std::string form;
  int steps_done = 0, steps_total = 0, blocks_done = 0, decode_done = 0;
  int affinity = -1;
  bool feasible = true;
  bool sunk = false;  // feasible only through the sunk-work deadband
  double best_remaining = 0;
  bool video() const { return kind == "video"; }
  bool finished_denoise() const { return steps_done >= steps_total; }
};

struct Gpus {
  std::vector<bool> free;
  std::vector<bool> image_only;
  // GPUs whose partial activations belong to a video suspended inside a solver step: other
  // videos do not take them (images may: a doorbell stopped the video for them)
  std::vector<std::string> reserved;
  std::string current;  // the video being placed
  std::vector<bool> decoding;  // a VAE decode runs on a side stream: no new video, images may overlap
  int count() const {
    int n = 0;
    for (bool f : free) n += f;
    return n;
  }
};

// first fully free aligned group of `size`, preferring `prefer` (no resize), then the most overlap
std::vector<int> pick_group(const Gpus& g, int size, const std::vector<int>& prefer, bool for_video) {
  const int n = static_cast<int>(g.free.size());
  auto usable = [&](int i) {
    return g.free[i] &&
           !(for_video && (g.image_only[i] || g.decoding[i] || (!g.reserved[i].empty() && g.reserved[i] != g.current)));
  };
  if (static_cast<int>(prefer.size()) == size) {
    bool ok = true;
    for (int i : prefer) ok = ok && i >= 0 && i < n && usable(i);
    if (ok) return prefer;
  }
  std::vector<int> best;
  int best_overlap = -1;
  for (const auto& grp : cluster_groups(n, size)) {
    bool ok = true;
    for (int i : grp) ok = ok && usable(i);
    if (!ok) continue;
    int overlap = 0;
    for (int i : grp) overlap += std::count(prefer.begin(), prefer.end(), i) > 0;
    if (overlap > best_overlap) {
      best = grp;
      best_overlap = overlap;
    }
  }
  return best;
}

// `claim` (optional): per GPU, the smallest laxity of the step-boundary videos that would
// resume there; within a placement tier the image takes the GPU with the largest claim, so
// it borrows from the video that can best afford to move (ties: the lowest index)
int pick_image_gpu(const Gpus& g, const std::string& placement, int affinity,
                   const std::vector<double>* claim = nullptr) {
  const int n = static_cast<int>(g.free.size());
  if (affinity >= 0) return affinity < n && g.free[affinity] ? affinity : -1;
  auto better = [&](int i, int cur) { return cur < 0 || (claim && (*claim)[i] > (*claim)[cur]); };
  int first = -1;
  // images prefer their reserved share when the cluster is partitioned
  for (int pass = 0; pass < 2 && first < 0; ++pass)
    for (int i = 0; i < n; ++i)
      if (g.free[i] && (pass == 1 || g.image_only[i]) && better(i, first)) first = i;
  if (placement != "pair_fit" || first < 0) return first;
  // pair_fit: take a GPU whose CFG-pair partner is already busy, so whole free pairs stay
  // available for videos; then one whose quad is partly busy
  for (int span : {2, 4}) {
    int pick = -1;
    for (int i = 0; i < n; ++i) {
      if (!g.free[i]) continue;
      const int base = i - i % span;
      bool partner_busy = false;
      for (int k = base; k < std::min(n, base + span); ++k)
        if (k != i && !g.free[k]) partner_busy = true;
      if (partner_busy && better(i, pick)) pick = i;
    }
    if (pick >= 0) return pick;
  }
  return first;
}

Json ints(const std::vector<int>& v) {
  Json a = Json::array();
  for (int i : v) a.push_back(i);
  return a;
}

}  // namespace

std::vector<Form> candidate_forms(const PolicyTraits& t, const ClusterCost& cost, const std::string& klass, int gpus,
                                  const Json& options) {
  return forms_for(resolve(t, options), cost, klass, gpus);
}

Json cluster_plan(const Json& state, const std::string& policy, const ClusterCost& cost, const Json& options,
                  PlanTrace* trace) {
  const PolicyTraits& traits = policy_traits(policy);
  const Settings s = resolve(traits, options);
  const PolicyTraits& t = s.t;
  const double now = state.at("now_ms").as_double();
  const int n = static_cast<int>(state.at("gpus").as_int());
  if (n <= 0) throw std::invalid_argument("gpus must be positive");
  Gpus g;
  g.free.assign(n, true);
  g.image_only.assign(n, false);
  g.reserved.assign(n, std::string());
  g.decoding.assign(n, false);
  if (state.contains("async_decoding")) {
    const auto& dec = state.at("async_decoding").as_array();
    if (static_cast<int>(dec.size()) != n) throw std::invalid_argument("async_decoding must list every GPU");
    for (int i = 0; i < n; ++i) g.decoding[i] = dec[i].as_bool();
  }
  if (state.contains("busy")) {
    const auto& busy = state.at("busy").as_array();
    if (static_cast<int>(busy.size()) != n) throw std::invalid_argument("busy must list every GPU");
    for (int i = 0; i < n; ++i) g.free[i] = !busy[i].as_bool();
  }
  // static image share
  int image_share = 0;
  if (t.partition_divisor > 0 || s.partition_image_gpus >= 0) {
    image_share = s.partition_image_gpus >= 0 ? s.partition_image_gpus : std::max(1, n / t.partition_divisor);
    const int video_min = std::max(1, t.fixed_degree > 0 ? t.fixed_degree : t.min_video_degree);
    image_share = std::max(0, std::min(image_share, n - video_min));
    for (int i = n - image_share; i < n; ++i) g.image_only[i] = true;
  }
  const int video_capacity = n - image_share;

  std::vector<Req> reqs;
  std::vector<Req> running;
  std::set<std::string> seen;
  // videos that still denoise (waiting, suspended or running): the load-adaptive choice
  // switches to the most GPU-efficient form once they could fill every CFG pair
  int video_load = 0;
  for (const auto& rj : state.at("requests").as_array()) {
    const std::string st = rj.str("status", "waiting");
    if (rj.str("kind", "") != "video" || (st != "waiting" && st != "suspended" && st != "running")) continue;
    video_load += rj.integer("steps_done", 0) < rj.integer("steps_total", cost.steps(rj.at("class").as_string()));
  }
  const bool throughput_mode = s.load_adaptive && video_load * 2 >= video_capacity;
  // widest aligned group free (and open to videos) when this plan starts
  int widest_free = 0;
  for (int d : {1, 2, 4, 8, 16, 32, 64}) {
    if (d > n) break;
    for (const auto& grp : cluster_groups(n, d)) {
      bool ok = true;
      for (int i : grp) ok = ok && g.free[i] && !g.image_only[i];
      if (ok) {
        widest_free = d;
        break;
      }
    }
  }
  auto efficient_only = [&](std::vector<Form> forms, const std::string& klass) {
    if (!throughput_mode || forms.size() < 2) return forms;
    const Form* eff = &forms.front();
    for (const auto& f : forms)
      if (cost.step_ms(klass, f) * f.degree() < cost.step_ms(klass, *eff) * eff->degree()) eff = &f;
    return std::vector<Form>{*eff};
  };
  // the candidate forms of a class depend only on the class within one plan
  std::map<std::string, std::vector<Form>> forms_cache;
  auto class_forms = [&](const std::string& klass) -> const std::vector<Form>& {
    auto it = forms_cache.find(klass);
    if (it == forms_cache.end()) it = forms_cache.emplace(klass, forms_for(s, cost, klass, video_capacity)).first;
    return it->second;
  };
  // remaining time including the dispatch overhead of the quanta still to run: one per solver
  // step (a step quantum stops early only on a doorbell), one per block quantum when the policy
  // runs fixed block quanta, one per decode chunk; images one
  auto remaining_q = [&](const Json& rj, const Form& f) {
    const double ms = cost.remaining_ms(rj, f);
    if (cost.overhead_ms() <= 0) return ms;
    const std::string k = rj.at("class").as_string();
    if (cost.kind(k) == "image") return ms + cost.overhead_ms();
    const int total = static_cast<int>(rj.integer("steps_total", cost.steps(k)));
    const int done = static_cast<int>(rj.integer("steps_done", 0));
    const int steps_left = std::max(0, total - done);
    long quanta = steps_left;
    if (t.blocks && s.quantum_blocks > 0 && steps_left > 0) {
      const int bps = cost.blocks_per_step(k), qb = s.quantum_blocks;
      const int first = std::max(0, bps - static_cast<int>(rj.integer("blocks_done", 0)));
      quanta = (first + qb - 1) / qb + static_cast<long>(steps_left - 1) * ((bps + qb - 1) / qb);
    }
    quanta += std::max(0, cost.decode_chunks(k) - static_cast<int>(rj.integer("decode_done", 0)));
    return ms + cost.overhead_ms() * static_cast<double>(quanta);
  };
  for (const auto& rj : state.at("requests").as_array()) {
    Req r;
    r.j = &rj;
    r.id = rj.at("request_id").as_string();
    if (!seen.insert(r.id).second) throw std::invalid_argument("duplicate request_id " + r.id);
    r.kind = rj.at("kind").as_string();
    r.klass = rj.at("class").as_string();
    if (r.kind != "video" && r.kind != "image") throw std::invalid_argument("kind must be video or image");
    r.status = rj.str("status", "waiting");
    r.arrival = rj.num("arrival_ms", 0.0);
    r.deadline = rj.num("deadline_ms", kInf);
    if (rj.contains("group"))
      for (const auto& i : rj.at("group").as_array()) r.group.push_back(static_cast<int>(i.as_int()));
    r.form = rj.str("form", r.group.empty() ? "" : "sp" + std::to_string(r.group.size()));
    r.steps_total = static_cast<int>(rj.integer("steps_total", cost.steps(r.klass)));
    r.steps_done = static_cast<int>(rj.integer("steps_done", 0));
    r.blocks_done = static_cast<int>(rj.integer("blocks_done", 0));
    r.decode_done = static_cast<int>(rj.integer("decode_done", 0));
    r.affinity = static_cast<int>(rj.integer("affinity", -1));
    if (r.status == "running") {
      running.push_back(r);
      continue;
    }
    if (r.status != "waiting" && r.status != "suspended") continue;
    // best-case finish on the whole cluster decides feasibility (on the form the video would
    // actually get when the load-adaptive choice is in throughput mode)
    if (r.video()) {
      double best = kInf;
      const auto forms = efficient_only(class_forms(r.klass), r.klass);
      int limit = video_capacity;
      if (s.feasibility_degree == "free" && !forms.empty()) limit = std::max(widest_free, forms.front().degree());
      for (const auto& f : forms)
        if (f.degree() <= limit) best = std::min(best, remaining_q(rj, f));
      if (!std::isfinite(best))
        for (const auto& f : forms) best = std::min(best, remaining_q(rj, f));
      if (!std::isfinite(best)) best = remaining_q(rj, Form{});
      r.best_remaining = best;
    } else {
      r.best_remaining = r.finished_denoise() ? cost.decode_ms(r.klass) : remaining_q(rj, Form{}) + cost.decode_ms(r.klass);
      if (!rj.contains("steps_done") && !(s.continuous_batch > 1)) r.best_remaining = cost.service_ms(r.klass);
    }
    r.feasible = now + r.best_remaining <= r.deadline;
    // sunk-work deadband: an in-flight video past half of its steps whose overrun is small
    // (at most 15 % of what remains, and at most 10 s) keeps its rank; demoting it would
    // discard the work already spent for a marginal miss
    if (!r.feasible && t.feasibility_guards && r.video() && r.status == "suspended" && r.steps_total > 0 &&
        2 * r.steps_done >= r.steps_total && std::isfinite(r.deadline) &&
        now + r.best_remaining - r.deadline <= std::min(10000.0, 0.15 * r.best_remaining)) {
      r.feasible = true;
      r.sunk = true;
    }
    reqs.push_back(r);
  }

  const bool image_boost = t.feasible_img_priority && t.elastic && !t.deadline_dp && !t.best_fit && !t.knapsack;
  auto key = [&](const Req& r) {
    // a late request is demoted behind feasible ones, unless it is short enough that serving
    // it now costs the others little (late_short_ms)
    const int late = (t.demote_late && !r.feasible && !(r.best_remaining <= s.late_short_ms)) ? 1 : 0;
    const int boost = (image_boost && !r.video() && r.feasible) ? 0 : 1;
    double primary = r.deadline;
    if (t.order == "srtf") primary = r.best_remaining;
    if (t.order == "fcfs") primary = r.arrival;
    // a suspended video that holds its group (no preemption) keeps its place first
    const int held = (t.hold_diffuse && r.status == "suspended" && r.video()) ? 0 : 1;
    return std::make_tuple(held, late, boost, primary, r.arrival, r.id);
  };
  std::stable_sort(reqs.begin(), reqs.end(), [&](const Req& a, const Req& b) { return key(a) < key(b); });
  if (trace) {
    for (const auto& r : reqs) {
      Json row = Json::object();
      row["request_id"] = r.id;
      row["feasible"] = r.feasible;
      row["laxity_ms"] = std::isfinite(r.deadline) ? r.deadline - now - r.best_remaining : 1e18;
      row["best_remaining_ms"] = r.best_remaining;
      if (r.sunk) row["sunk_work_deadband"] = true;
      trace->add(row);
    }
  }

  for (const auto& r : reqs)
    if (r.video() && r.status == "suspended" && r.blocks_done > 0)
      for (int i : r.group)
        if (i >= 0 && i < n && g.reserved[i].empty()) g.reserved[i] = r.id;

  Json assignments = Json::array();
  std::set<std::string> placed;
  struct Placed {
    std::string id;
    std::vector<int> group;
    Form form;
    size_t index;  // into assignments
    std::string klass;
    double deadline;
    const Json* j;
  };
  std::vector<Placed> placed_videos;

  auto take = [&](const std::vector<int>& grp) {
    for (int i : grp) g.free[i] = false;
  };
  auto give = [&](const std::vector<int>& grp) {
    for (int i : grp) g.free[i] = true;
  };

  auto video_quantum = [&](const Req& r, const Form& f, Json& a) {
    if (r.finished_denoise()) {
      a["quantum"] = "finish";
      const int chunks = cost.decode_chunks(r.klass);
      if (chunks > 1) a["decode_frames"] = t.blocks ? 1 : chunks - r.decode_done;
      return;
    }
    if (t.blocks && s.quantum_ms > 0) {
      // a preemption check about every quantum_ms of GPU work, never past the step boundary
      const int left = std::max(1, cost.blocks_per_step(r.klass) - r.blocks_done);
      const double blocks = std::floor(s.quantum_ms / cost.block_ms(r.klass, f));
      a["quantum"] = static_cast<int>(std::max(1.0, std::min(blocks, static_cast<double>(left))));
    } else if (t.blocks && s.quantum_blocks > 0) {
      a["quantum"] = s.quantum_blocks;
    } else {
      a["quantum"] = "step";
      if (t.rounds) a["steps"] = std::min(t.round_steps, r.steps_total - r.steps_done);
    }
  };

  auto emit_video = [&](const Req& r, const Form& f, const std::vector<int>& grp, const std::string& reason) {
    for (auto& holder : g.reserved)
      if (holder == r.id) holder.clear();
    Json a = Json::object();
    a["request_id"] = r.id;
    a["group"] = ints(grp);
    a["degree"] = static_cast<int>(grp.size());
    a["form"] = form_name(f);
    a["resize"] = !r.group.empty() && r.group != grp;
    a["reason"] = reason;
    video_quantum(r, f, a);
    take(grp);
    placed.insert(r.id);
    placed_videos.push_back({r.id, grp, f, assignments.size(), r.klass, r.deadline, r.j});
    assignments.push_back(a);
  };

  // ---- decode-only videos: a finished denoise decodes on one GPU (decode shrink) ----
  auto place_finish = [&](const Req& r) -> bool {
    g.current = r.id;
    std::vector<int> grp;
    Form f{1, 1, 1};
    if (t.hold_diffuse && !r.group.empty()) {
      grp = pick_group(g, static_cast<int>(r.group.size()), r.group, true);
      if (!r.form.empty()) f = parse_form(r.form);
    } else {
      std::vector<int> prefer;
      if (!r.group.empty()) prefer.push_back(r.group.front());
      grp = pick_group(g, 1, prefer, false);
    }
    if (grp.empty()) return false;
    emit_video(r, f, grp, t.hold_diffuse ? "finish-held" : "decode-shrink");
    return true;
  };

  std::vector<const Req*> videos, images;
  for (const auto& r : reqs) (r.video() ? videos : images).push_back(&r);

  // ---- feasibility-guard helpers -----------------------------------------------------
  std::map<std::string, int> min_degree_cache;
  auto min_feasible_degree = [&](const Req& o) -> int {  // 0: no form meets its deadline
    auto it = min_degree_cache.find(o.id);
    if (it != min_degree_cache.end()) return it->second;
    int d = 0;
    for (const auto& f : efficient_only(class_forms(o.klass), o.klass))
      if (now + remaining_q(*o.j, f) <= o.deadline) {
        d = f.degree();
        break;
      }
    if (d == 0 && o.sunk) {
      auto forms = class_forms(o.klass);
      if (!forms.empty()) d = forms.back().degree();
    }
    return min_degree_cache[o.id] = d;
  };
  auto video_free = [&]() {
    int c = 0;
    for (int i = 0; i < n; ++i) c += g.free[i] && !g.image_only[i] && !g.decoding[i];
    return c;
  };
  auto movable_after = [&](const Req& self, const Req& o, bool& after) {
    if (&o == &self) {
      after = true;
      return false;
    }
    return after && o.video() && !placed.count(o.id) && !o.finished_denoise() &&
           !(o.status == "suspended" && o.blocks_done > 0);
  };
  // feasible videos ranked after `self` that still get GPUs, greedily, out of `free_gpus`
  auto others_fitting = [&](const Req& self, int free_gpus) {
    int fit = 0;
    bool after = false;
    for (const auto& o : reqs) {
      if (!movable_after(self, o, after) || !o.feasible) continue;
      const int d = min_feasible_degree(o);
      if (d > 0 && d <= free_gpus) {
        free_gpus -= d;
        ++fit;
      }
    }
    return fit;
  };
  // GPUs the requests ranked after `self` still need: each video its minimal (feasible)
  // degree, each unplaced image one GPU
  auto others_need = [&](const Req& self) {
    int need = 0;
    bool after = false;
    for (const auto& o : reqs) {
      if (!o.video()) {
        if (&o != &self && !placed.count(o.id)) need += 1;
        continue;
      }
      if (!movable_after(self, o, after)) continue;
      int d = min_feasible_degree(o);
      if (d == 0) {
        auto forms = efficient_only(class_forms(o.klass), o.klass);
        d = forms.empty() ? 0 : forms.front().degree();
      }
      need += d;
    }
    return need;
  };
  // laxity claims of the step-boundary videos on the GPUs they would resume on
  std::vector<double> claim(n, kInf);
  if (t.feasibility_guards)
    for (const auto& r : reqs)
      if (r.video() && r.status == "suspended" && r.blocks_done == 0 && !r.group.empty() && !r.finished_denoise()) {
        const double lax = std::isfinite(r.deadline) ? r.deadline - now - r.best_remaining : 1e18;
        // a fold-eligible CFG2 video under fission continues on the conditional half of its
        // group: only that half is claimed, the companion half is the first choice for images
        size_t held = r.group.size();
        if (t.fission && r.j->flag("cfg_fold_eligible", false) && !r.form.empty() && parse_form(r.form).cfg == 2 &&
            held % 2 == 0)
          held /= 2;
        for (size_t k = 0; k < held; ++k)
          if (r.group[k] >= 0 && r.group[k] < n) claim[r.group[k]] = std::min(claim[r.group[k]], lax);
      }
  const std::vector<double>* claims = t.feasibility_guards ? &claim : nullptr;



  // ---- deadline knapsack (TetriServe / SBP-ESP / v1) over movable videos --------------
  std::map<std::string, Form> dp_choice;
  if (t.deadline_dp || t.knapsack) {
    int cap = 0;
    for (int i = 0; i < n; ++i) cap += g.free[i] && !g.image_only[i];
    struct Item {
      const Req* r;
      Form f;
      int w;
      double value;
    };
    std::vector<Item> items;
    for (const Req* r : videos) {
      if (r->finished_denoise()) continue;
      for (const auto& f : class_forms(r->klass)) {
        if (now + remaining_q(*r->j, f) <= r->deadline) {
          // unit value per request kept on track; v1 weighs urgency (small laxity first)
          double value = 1.0;
          if (t.knapsack) value += 1.0 / (1.0 + std::max(0.0, r->deadline - now) / 1000.0);
          items.push_back({r, f, f.degree(), value});
          break;  // minimal feasible degree
        }
      }
    }
    // 0/1 knapsack, max value then min weight
    const int W = cap;
    std::vector<double> best(W + 1, 0.0);
    std::vector<std::vector<int>> pick(W + 1);
    for (size_t k = 0; k < items.size(); ++k) {
      for (int w = W; w >= items[k].w; --w) {
        const double v = best[w - items[k].w] + items[k].value;
        if (v > best[w] + 1e-12) {
          best[w] = v;
          pick[w] = pick[w - items[k].w];
          pick[w].push_back(static_cast<int>(k));
        }
      }
    }
    int bw = 0;
    for (int w = 0; w <= W; ++w)
      if (best[w] > best[bw] + 1e-12) bw = w;
    for (int k : pick[bw]) dp_choice[items[k].r->id] = items[k].f;
  }

  auto fastest_fit = [&](const Req& r, std::vector<int>& grp_out, const std::vector<Form>* only = nullptr) -> Form {
    auto forms = only ? *only : class_forms(r.klass);
    Form best{0, 0, 0};
    double best_ms = kInf;
    for (const auto& f : forms) {
      auto grp = pick_group(g, f.degree(), r.group, true);
      if (grp.empty()) continue;
      const double ms = remaining_q(*r.j, f);
      if (ms < best_ms) {
        best_ms = ms;
        best = f;
        grp_out = grp;
      }
    }
    return best;
  };

  auto any_waiting_image_unplaced = [&]() {
    for (const Req* im : images)
      if (!placed.count(im->id)) return true;
    return false;
  };

  // ---- images ----------------------------------------------------------------------
  // time until a mid-step video reaches its step boundary if it resumes now
  auto time_to_boundary = [&](const std::string& owner) -> double {
    for (const auto& o : reqs)
      if (o.id == owner) {
        const Form f = o.form.empty() ? Form{1, static_cast<int>(o.group.size()), 1} : parse_form(o.form);
        return std::max(0, cost.blocks_per_step(o.klass) - o.blocks_done) * cost.block_ms(o.klass, f);
      }
    return kInf;
  };
  auto place_image = [&](const Req& r) -> bool {
    if (placed.count(r.id)) return true;
    // lazy block preemption: a new image does not take a GPU whose mid-step video can resume
    // now when waiting for that video's step boundary still meets the image's deadline
    std::vector<int> masked;
    if (t.blocks && s.lazy_preemption && r.affinity < 0 && !r.j->contains("steps_done") && std::isfinite(r.deadline)) {
      const double slack = r.deadline - now - r.best_remaining;
      for (int i = 0; i < n; ++i) {
        if (!g.free[i] || g.reserved[i].empty()) continue;
        bool resumable = true;
        for (const auto& o : reqs)
          if (o.id == g.reserved[i])
            for (int k : o.group) resumable = resumable && k >= 0 && k < n && g.free[k];
        if (resumable && slack > 0 && time_to_boundary(g.reserved[i]) <= slack) masked.push_back(i);
      }
    }
    for (int i : masked) g.free[i] = false;
    const int gpu = pick_image_gpu(g, t.image_placement, r.affinity, claims);
    for (int i : masked) g.free[i] = true;
    if (gpu < 0) return false;
    Json a = Json::object();
    a["request_id"] = r.id;
    a["group"] = ints({gpu});
    a["degree"] = 1;
    a["form"] = "sp1";
    a["resize"] = false;
    // continuous batching: same-class waiting images join while every member keeps its deadline
    // late_image_batching: an image that can no longer make its deadline is packed into a
    // continuous batch (fewer GPUs for work that is late anyway) even when the policy runs
    // on-time images atomically
    const bool late_cb = s.late_image_batching && !r.feasible && s.continuous_batch <= 1;
    const bool cb = (s.continuous_batch > 1 || late_cb) && cost.klass(r.klass).contains("batch_step_ms");
    const bool ab = !cb && s.image_batch > 1 && cost.klass(r.klass).contains("batch_ms") && g.count() <= 1;
    if (cb || ab) {
      std::vector<const Req*> members{&r};
      auto joins = [&](const Req* other) {
        return other != &r && !placed.count(other->id) && (s.t.sequence_packing || other->klass == r.klass) &&
               (other->affinity < 0 || other->affinity == gpu) && (!late_cb || !other->feasible);
      };
      int cap = cb ? (late_cb ? 8 : s.continuous_batch) : s.image_batch;
      if (cb) {
        // work-conserving: while GPUs that no waiting video needs are idle, the waiting images
        // spread over them (fewer members per GPU, shorter rounds) instead of queueing on one
        int pending = 1;
        for (const Req* other : images) pending += joins(other);
        int video_need = 0;
        for (const Req* v : videos)
          if (!placed.count(v->id) && !v->finished_denoise() && v->feasible) video_need += min_feasible_degree(*v);
        const int spare = std::max(1, g.count() - video_need);
        cap = std::min(cap, std::max(1, (pending + spare - 1) / spare));
      }
      for (const Req* other : images) {
        if (static_cast<int>(members.size()) >= cap) break;
        if (!joins(other)) continue;
        std::vector<const Json*> js;
        for (auto* m : members) js.push_back(m->j);
        js.push_back(other->j);
        // every member, the joining one included, keeps its deadline; a mixed batch is priced
        // on the table of its largest class whichever member anchors it
        double round_ms = cb ? cost.continuous_batch_step_ms(js, s.t.sequence_packing, r.klass) : 0.0;
        std::vector<const Req*> all = members;
        all.push_back(other);
        // without bubble-free admission a member's prepare and finish stall the whole round;
        // bubble-free batches overlap them with the other members' denoising
        if (cb && !s.t.bubble_free)
          for (auto* m : all) {
            const Json& kc = cost.klass(m->klass);
            if (!m->j->flag("prepared", m->steps_done > 0)) round_ms += kc.num("prepare_ms", 0.0);
            if (m->steps_done + 1 >= m->steps_total) round_ms += kc.num("finish_ms", 0.0);
          }
        bool ok = true;
        for (auto* m : all) {
          const int left = m->steps_total - m->steps_done;
          const double ms = cb ? left * round_ms + cost.decode_ms(m->klass)
                               : cost.batch_ms(r.klass, static_cast<int>(js.size()));
          if (m->feasible && now + ms > m->deadline) ok = false;
        }
        if (ok) members.push_back(other);
      }
      if (members.size() > 1 || cb) {
        Json b = Json::array();
        for (auto* m : members) {
          b.push_back(m->id);
          placed.insert(m->id);
        }
        a["batch"] = b;
      }
      a["quantum"] = cb ? "continuous_batch" : "atomic";
      a["reason"] = cb ? "continuous-batch" : (members.size() > 1 ? "image-batch" : t.image_placement);
      if (cb) {
        a["sequence_packing"] = s.t.sequence_packing;
        a["bubble_free"] = s.t.bubble_free;
      }
    } else {
      a["quantum"] = r.finished_denoise() && r.j->contains("steps_done") ? "finish" : "atomic";
      a["reason"] = t.image_placement;
    }
    g.free[gpu] = false;
    placed.insert(r.id);
    assignments.push_back(a);
    return true;
  };

  // ---- main pass in rank order -------------------------------------------------------
  for (const auto& r : reqs) {
    if (placed.count(r.id)) continue;
    if (!r.video()) {
      place_image(r);
      continue;
    }
    if (r.finished_denoise()) {
      place_finish(r);
      continue;
    }
    g.current = r.id;
    // load-adaptive form choice: when the videos in the system could fill every CFG pair,
    // throughput decides and each video takes the form with the least GPU time per step;
    // otherwise the usual feasible-minimal choice (and widening) keeps latency low
    const std::vector<Form> forms = efficient_only(class_forms(r.klass), r.klass);
    if (forms.empty()) continue;
    // CFG fission (approximate policies): a video whose next step runs folded (conditional
    // branch only, the guidance delta reused) continues on the conditional half of its CFG2
    // group; the unconditional half is free for other work this round
    if (t.fission && r.j->flag("cfg_fold_eligible", false) && !r.group.empty() && !r.form.empty() &&
        r.blocks_done == 0) {
      const Form f = parse_form(r.form);
      if (f.cfg == 2 && r.group.size() % 2 == 0) {
        const std::vector<int> half(r.group.begin(), r.group.begin() + r.group.size() / 2);
        auto grp = pick_group(g, static_cast<int>(half.size()), half, true);
        if (grp == half) {
          emit_video(r, Form{1, f.sp, f.ring}, grp, "fission");
          assignments.at(assignments.size() - 1)["fold"] = true;
          continue;
        }
      }
    }
    // inside a solver step the request's partial activations live on its group, sharded
    // for its form: it resumes there (or waits), never on other GPUs
    if (r.status == "suspended" && r.blocks_done > 0 && !r.group.empty()) {
      auto grp = pick_group(g, static_cast<int>(r.group.size()), r.group, true);
      if (grp == r.group) emit_video(r, r.form.empty() ? forms.front() : parse_form(r.form), grp, "mid-step");
      continue;
    }
    if (t.hold_diffuse && r.status == "suspended" && !r.group.empty()) {
      // run-to-completion baselines resume on exactly their GPUs
      auto grp = pick_group(g, static_cast<int>(r.group.size()), r.group, true);
      if (grp == r.group) emit_video(r, r.form.empty() ? forms.front() : parse_form(r.form), grp, "held");
      continue;
    }
    if (t.fixed_degree > 0) {
      auto grp = pick_group(g, t.fixed_form.degree(), r.group, true);
      if (!grp.empty()) emit_video(r, t.fixed_form, grp, "fixed");
      continue;
    }
    if (t.deadline_dp || t.knapsack) {
      auto it = dp_choice.find(r.id);
      if (it != dp_choice.end()) {
        auto grp = pick_group(g, it->second.degree(), r.group, true);
        if (!grp.empty()) {
          emit_video(r, it->second, grp, "knapsack");
          continue;
        }
      }
      continue;  // leftovers handled below
    }
    // minimal form that meets the deadline, else the fastest that fits
    Form chosen{0, 0, 0};
    std::vector<int> grp;
    std::string reason;
    const int free_now = video_free();
    const int d_min = forms.front().degree();
    bool guarded = false, migration_held = false;
    for (const auto& f : forms) {
      const double rem = remaining_q(*r.j, f);
      if (now + rem * (1.0 + s.feasible_margin) > r.deadline) continue;
      auto cand = pick_group(g, f.degree(), r.group, true);
      if (cand.empty()) continue;
      if (t.feasibility_guards) {
        // multi-video guard: widening to save this deadline may not cost two others theirs
        if (f.degree() > d_min && others_fitting(r, free_now - d_min) - others_fitting(r, free_now - f.degree()) >= 2) {
          guarded = true;
          continue;
        }
        // migration guard: a prepared video does not move to another group of its size when
        // the reshard makes it late; it waits for its own GPUs
        if (r.status == "suspended" && !r.group.empty() && cand != r.group &&
            static_cast<int>(r.group.size()) == f.degree() && now + rem + cost.resize_ms() > r.deadline) {
          migration_held = true;
          continue;
        }
      }
      chosen = f;
      grp = cand;
      reason = t.best_fit ? "best-fit" : "feasible-min";
      break;
    }
    if (chosen.degree() == 0 && guarded) {
      auto cand = pick_group(g, d_min, r.group, true);
      if (!cand.empty()) {
        chosen = forms.front();
        grp = cand;
        reason = "multi-video-guard";
      }
    }
    if (chosen.degree() == 0 && migration_held) continue;
    if (chosen.degree() == 0) {
      if (t.best_fit) {
        // largest group that fits
        for (auto it = forms.rbegin(); it != forms.rend(); ++it) {
          auto cand = pick_group(g, it->degree(), r.group, true);
          if (!cand.empty()) {
            chosen = *it;
            grp = cand;
            reason = "best-fit-largest";
            break;
          }
        }
      } else {
        chosen = fastest_fit(r, grp, &forms);
        reason = r.feasible ? "fastest-fit" : "late-fastest";
      }
    }
    if (chosen.degree() == 0) continue;
    // widen while the per-GPU efficiency stays above the threshold and no image is starved
    // (nor, with the guards, any feasible video); `grp` is not taken until emit_video
    if (t.widen > 0 && !t.best_fit) {
      for (const auto& f : forms) {
        if (f.degree() <= chosen.degree()) continue;
        const double base_work = cost.step_ms(r.klass, chosen) * chosen.degree();
        const double wide_work = cost.step_ms(r.klass, f) * f.degree();
        if (base_work / wide_work < t.widen) break;
        if (!s.widen_past_images && any_waiting_image_unplaced()) break;
        if (t.feasibility_guards &&
            others_fitting(r, free_now - chosen.degree()) - others_fitting(r, free_now - f.degree()) >= 1)
          break;
        auto cand = pick_group(g, f.degree(), r.group, true);
        if (cand.empty()) continue;
        chosen = f;
        grp = cand;
        reason = "widened";
      }
    }
    // idle widening: below the threshold, a faster wider form still takes GPUs that neither
    // the requests ranked after this one nor a waiting image would use this round
    if (t.idle_widening && !t.best_fit && !throughput_mode && !any_waiting_image_unplaced()) {
      const int need = others_need(r);
      for (const auto& f : forms) {
        if (f.degree() <= chosen.degree()) continue;
        if (f.degree() + need > free_now) break;
        if (cost.step_ms(r.klass, f) >= cost.step_ms(r.klass, chosen)) continue;
        auto cand = pick_group(g, f.degree(), r.group, true);
        if (cand.empty()) continue;
        chosen = f;
        grp = cand;
        reason = "idle-widened";
      }
    }
    emit_video(r, chosen, grp, reason);
  }

  // ---- knapsack leftovers: widest-first in EDF order to requests no size saves -------
  if (t.deadline_dp || t.knapsack) {
    for (const Req* r : videos) {
      if (placed.count(r->id) || r->finished_denoise()) continue;
      if (r->status == "suspended" && r->blocks_done > 0 && !r->group.empty()) continue;  // mid-step: own group only
      g.current = r->id;
      std::vector<int> grp;
      auto forms = class_forms(r->klass);
      for (auto it = forms.rbegin(); it != forms.rend(); ++it) {
        grp = pick_group(g, it->degree(), r->group, true);
        if (!grp.empty()) {
          emit_video(*r, *it, grp, "knapsack-leftover");
          break;
        }
      }
    }
  }

  // ---- surplus redistribution (EDF-BF) / idle widening (knapsack baselines) ----------
  if ((t.best_fit || t.deadline_dp) && !any_waiting_image_unplaced()) {
    bool grew = true;
    while (grew) {
      grew = false;
      for (auto& pv : placed_videos) {
        Json& a = assignments.at(pv.index);
        if (a.at("quantum").is_string() && a.at("quantum").as_string() == "finish") continue;
        // a request inside a solver step (or pinned to its group) keeps its group and form
        const std::string why = a.at("reason").as_string();
        if (why == "mid-step" || why == "held" || why == "fixed" || why == "fission") continue;
        g.current = pv.id;
        auto forms = class_forms(pv.klass);
        for (const auto& f : forms) {
          if (f.degree() <= pv.form.degree()) continue;
          give(pv.group);
          auto cand = pick_group(g, f.degree(), pv.group, true);
          if (cand.empty() || cost.step_ms(pv.klass, f) >= cost.step_ms(pv.klass, pv.form)) {
            take(pv.group);
            continue;
          }
          take(cand);
          pv.group = cand;
          pv.form = f;
          a["group"] = ints(cand);
          a["degree"] = f.degree();
          a["form"] = form_name(f);
          a["reason"] = "surplus";
          grew = true;
          break;
        }
      }
    }
  }

  // ---- lockstep pairing: an unplaced video joins a placed one on its group -----------
  if (s.pairing && t.elastic) {
    for (const Req* r : videos) {
      if (placed.count(r->id) || r->finished_denoise()) continue;
      for (auto& pv : placed_videos) {
        Json& a = assignments.at(pv.index);
        if (a.contains("pair") || !a.at("quantum").is_string() || a.at("quantum").as_string() != "step") continue;
        const double alone = cost.step_ms(pv.klass, pv.form);
        const double paired = cost.pair_ms(pv.klass, r->klass, pv.form);
        if (paired >= alone + cost.step_ms(r->klass, pv.form)) continue;
        const int left = static_cast<int>(pv.j->integer("steps_total", cost.steps(pv.klass)) - pv.j->integer("steps_done", 0));
        if (now + left * paired > pv.deadline) continue;
        a["pair"] = r->id;
        Json b = Json::object();
        b["request_id"] = r->id;
        b["group"] = ints(pv.group);
        b["degree"] = pv.form.degree();
        b["form"] = form_name(pv.form);
        b["quantum"] = "step";
        b["pair"] = pv.id;
        b["resize"] = !r->group.empty() && r->group != pv.group;
        b["reason"] = "paired";
        placed.insert(r->id);
        assignments.push_back(b);
        break;
      }
    }
  }

  Json out = Json::object();
  out["assignments"] = assignments;

  // ---- sub-step preemption of running video groups for waiting images -----------------
  Json preempt = Json::array();
  size_t skips = 0;
  if (t.blocks && s.preempt && !running.empty()) {
    std::vector<ImageDemand> demand;
    for (const Req* im : images) {
      if (placed.count(im->id)) continue;
      demand.push_back({im->affinity, im->deadline, im->best_remaining});
    }
    if (!demand.empty()) {
      std::vector<RunningGroup> groups;
      std::set<int> claimed;  // the two requests of a lockstep pair share one group: list it once
      for (const auto& r : running) {
        if (!r.video() || r.group.empty()) continue;
        bool shared = false;
        for (int gpu : r.group) shared = shared || claimed.count(gpu) > 0;
        if (shared) continue;
        claimed.insert(r.group.begin(), r.group.end());
        Form f = r.form.empty() ? Form{1, static_cast<int>(r.group.size()), 1} : parse_form(r.form);
        const double bms = cost.block_ms(r.klass, f);
        const double elapsed = std::max(0.0, now - r.j->num("quantum_started_ms", now));
        auto timing = estimate_preemption_timing(bms, cost.blocks_per_step(r.klass), r.blocks_done, elapsed,
                                                 std::max(1, s.check_blocks), 1, f.sp > 1);
        groups.push_back({r.id, r.group, timing.stop_ms, timing.remaining_ms, cost.resume_ms(r.klass),
                          r.j->flag("rung", false)});
      }
      auto sel = select_deadline_preemption(now, demand, groups);
      for (const auto& id : sel.selected) preempt.push_back(id);
      skips = sel.deadline_skips;
    }
  }
  out["preempt"] = preempt;
  out["deadline_skips"] = static_cast<int>(skips);
  return out;
}

// ---------------------------------------------------------------------------------------
// Block preemption (sub-step, through doorbells).
//
// Decision rules; the golden fixture's "preemption" section pins them on generated cases,
// ties included.
//
// Timing of a running group.  A rung group stops at its next doorbell check, which comes
//   every check_blocks x blocks_per_iteration blocks, or twice that when the group agrees on
//   the flag one checkpoint late.  Unrung, it runs to its step boundary: the blocks still to
//   run less the time already spent, and never less than one block.
//
// A stop saves an image when waiting for the group's boundary makes the image late and the
//   earlier of the stop and the boundary lets it finish on time.
//
// Freeing GPUs for waiting images (select_preemption_groups):
//   1. Groups that already rang, and groups that hold a GPU some image is pinned to, stop
//      anyway; those that did not ring yet are selected, in input order.
//   2. Their GPUs that no image is pinned to go to the images that take any GPU.
//   3. If such images remain without a GPU, more groups are chosen so that they free at
//      least that many GPUs (or all they have), displacing the least GPU time, where a group
//      displaces |group| x (min(stop, remaining) + resume).  Candidate sets are ordered by
//      displaced time (summed in input order), then by GPUs freed, then by the number of
//      groups, then by the position of their last group in the input, comparing from the
//      back (the set whose last member comes earlier wins).  The chosen groups follow the
//      pinned ones, in input order.
//
// Matching images to groups by deadline (select_deadline_preemption):
//   Images are served in deadline order; among equal deadlines an image pinned to a GPU goes
//   first.  A group can serve an image when it holds a GPU that no earlier image was promised
//   and that the image may use; the first such GPU of the group is the one promised.  The
//   image's window is tight when its deadline lies between 0.85x and 1.35x of its service
//   time from now; a tight image tolerates a rung group overrunning its deadline by
//   max(1.5 x stop, 120 ms).
//   a) A group that already rang and responds in time (within that tolerance) takes the
//      image, the earliest responder first.
//   b) Otherwise, if waiting for the earliest response among the usable groups is late, a
//      group is rung: one whose early stop saves the image, or, failing that and only for a
//      tight image, one that stops before its boundary and within the tolerance.  Among the
//      candidates the least displaced time wins, then the narrower group, then the earlier.
//   c) An image served neither way counts as a deadline skip.

PreemptionTiming estimate_preemption_timing(double block_ms, int blocks_total, int blocks_done, double elapsed_ms,
                                            int check_blocks, int blocks_per_iteration, bool delayed_group_check) {
  const bool sane = block_ms > 0 && std::isfinite(block_ms) && blocks_total > 0 && blocks_done >= 0 &&
                    elapsed_ms >= 0 && check_blocks > 0 && blocks_per_iteration > 0;
  if (!sane) throw std::invalid_argument("invalid block preemption timing");
  const int blocks_per_check = check_blocks * blocks_per_iteration;
  const double checks_to_stop = delayed_group_check ? 2 : 1;
  const int blocks_left = blocks_total > blocks_done ? blocks_total - blocks_done : 0;
  PreemptionTiming out;
  out.stop_ms = block_ms * blocks_per_check * checks_to_stop;
  out.remaining_ms = std::max(block_ms, blocks_left * block_ms - elapsed_ms);
  return out;
}

namespace {

void require_preemption_inputs(double now_ms, double deadline_ms, double service_ms, double stop_ms,
                               double boundary_ms) {
  const double all[] = {now_ms, deadline_ms, service_ms, stop_ms, boundary_ms};
  if (!std::all_of(std::begin(all), std::end(all), [](double v) { return std::isfinite(v); }))
    throw std::invalid_argument("non-finite preemption input");
  if (std::min({now_ms, service_ms, stop_ms, boundary_ms}) < 0)
    throw std::invalid_argument("negative preemption input");
}

}  // namespace

bool preemption_converts_deadline(double now_ms, double deadline_ms, double service_ms, double stop_ms,
                                  double boundary_ms) {
  require_preemption_inputs(now_ms, deadline_ms, service_ms, stop_ms, boundary_ms);
  const double finish_waiting = now_ms + boundary_ms + service_ms;
  const double finish_stopping = now_ms + std::min(stop_ms, boundary_ms) + service_ms;
  return finish_waiting > deadline_ms && finish_stopping <= deadline_ms;
}

namespace {

void require_disjoint_groups(const std::vector<RunningGroup>& running) {
  std::set<std::string> seen_ids;
  std::set<int> seen_gpus;
  for (const auto& g : running) {
    const bool named = !g.request_id.empty() && seen_ids.insert(g.request_id).second && !g.group.empty();
    if (!named) throw std::invalid_argument("invalid running group");
    const double times[] = {g.stop_ms, g.remaining_ms, g.resume_ms};
    for (double v : times)
      if (!std::isfinite(v) || v < 0) throw std::invalid_argument("invalid running group timing");
    for (int gpu : g.group)
      if (gpu < 0 || !seen_gpus.insert(gpu).second) throw std::invalid_argument("running groups must be disjoint");
  }
}

// GPU time lost when a group stops now and later resumes: every GPU of the group idles for
// the stop (or the boundary, if sooner) and then pays the resume.
double displaced_gpu_ms(const RunningGroup& g) {
  return g.group.size() * (std::min(g.stop_ms, g.remaining_ms) + g.resume_ms);
}

// Least displaced GPU time that frees at least `need` GPUs out of `pool` (indices into
// `running`), by the order stated above.  A table over (groups considered, GPUs freed)
// holds the best set for each exact GPU count; a set that leaves out the newest group wins
// every tie against one that takes it, which is the "last member earlier" rule.
std::vector<size_t> cheapest_cover(const std::vector<RunningGroup>& running, const std::vector<size_t>& pool,
                                   int need) {
  struct Best {
    double cost = std::numeric_limits<double>::infinity();
    int groups = 0;
    bool took = false;
  };
  int total = 0;
  for (size_t idx : pool) total += static_cast<int>(running[idx].group.size());
  const size_t n = pool.size();
  std::vector<std::vector<Best>> best(n + 1, std::vector<Best>(total + 1));
  best[0][0].cost = 0;
  for (size_t i = 1; i <= n; ++i) {
    const RunningGroup& g = running[pool[i - 1]];
    const int w = static_cast<int>(g.group.size());
    const double d = displaced_gpu_ms(g);
    for (int c = 0; c <= total; ++c) {
      Best keep = best[i - 1][c];
      keep.took = false;
      best[i][c] = keep;
      if (c < w || !std::isfinite(best[i - 1][c - w].cost)) continue;
      const Best& from = best[i - 1][c - w];
      const double cost = from.cost + d;
      const int groups = from.groups + 1;
      const bool better = cost < keep.cost || (cost == keep.cost && groups < keep.groups);
      if (better) best[i][c] = Best{cost, groups, true};
    }
  }
  int pick = need;
  for (int c = need + 1; c <= total; ++c)
    if (best[n][c].cost < best[n][pick].cost) pick = c;
  std::vector<size_t> chosen;
  for (size_t i = n, c = static_cast<size_t>(pick); i > 0; --i) {
    if (!best[i][c].took) continue;
    chosen.push_back(pool[i - 1]);
    c -= running[pool[i - 1]].group.size();
  }
  std::reverse(chosen.begin(), chosen.end());
  return chosen;
}

}  // namespace

std::vector<std::string> select_preemption_groups(const std::vector<int>& affinities,
                                                  const std::vector<RunningGroup>& running) {
  require_disjoint_groups(running);
  if (std::any_of(affinities.begin(), affinities.end(), [](int a) { return a < -1; }))
    throw std::invalid_argument("invalid image affinity");
  const std::set<int> pinned_gpus = [&] {
    std::set<int> s;
    for (int a : affinities)
      if (a >= 0) s.insert(a);
    return s;
  }();
  const size_t any_gpu_images = static_cast<size_t>(std::count(affinities.begin(), affinities.end(), -1));

  std::vector<std::string> out;
  std::set<int> stopping_gpus;
  std::vector<size_t> pool;  // groups that may keep running
  for (size_t i = 0; i < running.size(); ++i) {
    const RunningGroup& g = running[i];
    const bool holds_pinned =
        std::any_of(g.group.begin(), g.group.end(), [&](int gpu) { return pinned_gpus.count(gpu) > 0; });
    if (!g.rung && !holds_pinned) {
      pool.push_back(i);
      continue;
    }
    stopping_gpus.insert(g.group.begin(), g.group.end());
    if (!g.rung) out.push_back(g.request_id);
  }
  const size_t free_for_any = static_cast<size_t>(
      std::count_if(stopping_gpus.begin(), stopping_gpus.end(), [&](int gpu) { return !pinned_gpus.count(gpu); }));
  if (any_gpu_images <= free_for_any) return out;
  int pool_gpus = 0;
  for (size_t i : pool) pool_gpus += static_cast<int>(running[i].group.size());
  const int shortfall = static_cast<int>(std::min<size_t>(any_gpu_images - free_for_any, pool_gpus));
  if (shortfall == 0) return out;
  for (size_t i : cheapest_cover(running, pool, shortfall)) out.push_back(running[i].request_id);
  return out;
}

namespace {

// The candidate that displaces the least GPU time; the narrower group on equal time; the
// first offered on a full tie.
class CheapestStop {
 public:
  void offer(int index, double cost, size_t width) {
    const bool better = index_ < 0 || cost < cost_ || (cost == cost_ && width < width_);
    if (!better) return;
    index_ = index;
    cost_ = cost;
    width_ = width;
  }
  int index() const { return index_; }

 private:
  int index_ = -1;
  double cost_ = 0;
  size_t width_ = 0;
};

}  // namespace

DeadlinePreemption select_deadline_preemption(double now_ms, const std::vector<ImageDemand>& waiting,
                                              const std::vector<RunningGroup>& running) {
  require_disjoint_groups(running);
  for (const auto& img : waiting) {
    if (img.affinity < -1) throw std::invalid_argument("invalid image affinity");
    require_preemption_inputs(now_ms, img.deadline_ms, img.service_ms, 0, 0);
  }
  std::vector<const ImageDemand*> queue;
  for (const auto& img : waiting) queue.push_back(&img);
  std::stable_sort(queue.begin(), queue.end(), [](const ImageDemand* a, const ImageDemand* b) {
    if (a->deadline_ms != b->deadline_ms) return a->deadline_ms < b->deadline_ms;
    return a->affinity >= 0 && b->affinity < 0;
  });

  std::vector<bool> rung(running.size());
  for (size_t i = 0; i < running.size(); ++i) rung[i] = running[i].rung;
  std::set<int> promised;
  DeadlinePreemption out;
  for (const ImageDemand* img : queue) {
    // the GPU of group i this image would get, or -1
    auto usable_gpu = [&](size_t i) {
      for (int gpu : running[i].group) {
        if (promised.count(gpu)) continue;
        if (img->affinity < 0 || gpu == img->affinity) return gpu;
      }
      return -1;
    };
    const bool tight =
        img->deadline_ms >= now_ms + 0.85 * img->service_ms && img->deadline_ms - now_ms <= 1.35 * img->service_ms;
    auto tolerance = [&](size_t i) { return tight ? std::max(1.5 * running[i].stop_ms, 120.0) : 0.0; };
    auto in_time = [&](size_t i, double response) {
      return now_ms + response + img->service_ms <= img->deadline_ms + tolerance(i);
    };

    // a) an already-rung group responding in time
    double earliest = std::numeric_limits<double>::infinity();
    int responder = -1;
    double responder_at = std::numeric_limits<double>::infinity();
    for (size_t i = 0; i < running.size(); ++i) {
      if (usable_gpu(i) < 0) continue;
      const RunningGroup& g = running[i];
      const double response = rung[i] ? std::min(g.stop_ms, g.remaining_ms) : g.remaining_ms;
      earliest = std::min(earliest, response);
      if (rung[i] && in_time(i, response) && response < responder_at) {
        responder = static_cast<int>(i);
        responder_at = response;
      }
    }
    if (responder >= 0) {
      promised.insert(usable_gpu(static_cast<size_t>(responder)));
      continue;
    }

    // b) ring a group, only if waiting for the earliest response is late
    CheapestStop pick;
    const bool waiting_is_late =
        std::isfinite(earliest) && now_ms + earliest + img->service_ms > img->deadline_ms;
    if (waiting_is_late) {
      for (size_t i = 0; i < running.size(); ++i) {
        const RunningGroup& g = running[i];
        if (rung[i] || usable_gpu(i) < 0) continue;
        if (preemption_converts_deadline(now_ms, img->deadline_ms, img->service_ms, g.stop_ms, g.remaining_ms))
          pick.offer(static_cast<int>(i), displaced_gpu_ms(g), g.group.size());
      }
      if (pick.index() < 0 && tight) {
        for (size_t i = 0; i < running.size(); ++i) {
          const RunningGroup& g = running[i];
          if (rung[i] || usable_gpu(i) < 0 || g.stop_ms >= g.remaining_ms) continue;
          if (in_time(i, std::min(g.stop_ms, g.remaining_ms)))
            pick.offer(static_cast<int>(i), displaced_gpu_ms(g), g.group.size());
        }
      }
    }
    if (pick.index() < 0) {
      ++out.deadline_skips;  // c)
      continue;
    }
    const size_t chosen = static_cast<size_t>(pick.index());
    out.selected.push_back(running[chosen].request_id);
    rung[chosen] = true;
    promised.insert(usable_gpu(chosen));
  }
  return out;
}

}  // namespace ds
