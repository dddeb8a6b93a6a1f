// Golden decision fixture: the simulator's outcome for every registered policy on a seeded
// mixed trace, the planner's assignments on a set of fixed cluster states, and the online
// selector's decisions on fixed queues, the resolution of every way a policy name can be
// written, and the block-preemption selectors' decisions on generated cases (ties included),
// compared against tests/fixtures/control-golden.json.
// Any change of a decision rule shows up here as a diff; after an intended change, rebuild
// the fixture with DS_UPDATE_GOLDEN=1 and review the diff.  (The reference keeps such a
// fixture for its control rules: tests/fixtures/control-baseline.json.)
#include <cmath>
#include <cstdint>
#include <initializer_list>
#include <vector>
#include <cstdlib>
#include <fstream>
#include <sstream>

#include "check.hpp"
#include "ds/dispatch.hpp"
#include "ds/planner.hpp"
#include "ds/policy.hpp"
#include "ds/sim.hpp"
#include "ds/study.hpp"
#include "ds/workload.hpp"

using namespace ds;

namespace {

Json profile() {
  return Json::parse(R"({"links":{"default_gbps":700,"default_latency_ms":0.02},
   "sp_efficiency":{"2":0.97,"4":0.94,"8":0.88},"quantum_overhead_ms":0,"resize_ms":20,
   "classes":{
    "vid":{"kind":"video","steps":10,"blocks_per_step":30,"heads":12,"step_compute_ms":800,
           "comm_mb_per_step":20000,"collectives_per_step":240,"cfg_exchange_mb":4,"decode_ms":100,"decode_chunks":2},
    "img":{"kind":"image","steps":28,"tokens":1024,"step_ms":12,"service_ms":400,"decode_ms":50,
           "batch_ms":{"1":400,"2":520,"4":800},"batch_step_ms":{"1":12,"2":16,"4":26,"8":46}},
    "big":{"kind":"image","steps":28,"tokens":4096,"step_ms":40,"service_ms":1300,"decode_ms":180,
           "batch_ms":{"1":1300,"2":2300},"batch_step_ms":{"1":40,"2":74,"4":142,"8":280}}}})");
}

double round6(double x) { return std::round(x * 1e6) / 1e6; }

// Deterministic case generator for the decision sections below (a 64-bit LCG, so the cases
// never depend on the standard library's distributions).
struct CaseGen {
  uint64_t s;
  explicit CaseGen(uint64_t seed) : s(seed * 2862933555777941757ull + 3037000493ull) {}
  uint64_t next() {
    s = s * 6364136223846793005ull + 1442695040888963407ull;
    return s >> 17;
  }
  int below(int n) { return static_cast<int>(next() % static_cast<uint64_t>(n)); }
  template <class T>
  T pick(std::initializer_list<T> v) { return *(v.begin() + below(static_cast<int>(v.size()))); }
};

Json name_resolution() {
  // every way a policy name can be written: registered ids, legacy aliases, retired names,
  // parameterised families in both spellings, malformed forms and unknown names
  std::vector<std::string> names;
  const Json catalog = policy_catalog();
  for (const auto& p : catalog.as_array()) names.push_back(p.at("id").as_string());
  for (const char* n : {"heterodit_exact", "knapsack_dp", "heterodit_v5", "step_elastic", "block_elastic",
                        "round_elastic", "heterodit_approx", "heterodit_v3", "ablation_tiered", "ablation_2d_usp",
                        "static_partition", "vanilla_xdit", "tridentserve_stage", "vllm_omni", "gf_dit",
                        "genserve_40gb", "xdit", "xdit_sp2", "xdit-sp8", "xdit-cfg2sp4", "static-sp1", "static_sp2",
                        "static_cfg2sp2", "static-u2r2", "static_u2r4", "block-cfg2", "block_cfg2sp4", "block-sp4",
                        "fold-cfg2", "fold-sp2", "fold_cfg2", "approx-cfg2sp2", "approx_cfg2sp2", "static-bogus",
                        "static_bogus", "block-", "static-cfg3", "static-u2r1x", "nope", "", "ditserve_",
                        "static_cfg2-sp2", "block-sp2_x", "static-sp32", "xdit-u1r2", "STATIC-sp2", "xdit-sp2",
                        "fold-cfg2sp3", "approx-cfg2sp3", "xdit-cfg2"})
    names.push_back(n);
  Json out = Json::object();
  for (const auto& n : names) {
    Json r = Json::object();
    try {
      r["legacy_alias"] = legacy_policy_alias(n);
    } catch (const std::exception& e) {
      r["legacy_alias_error"] = std::string(e.what());
    }
    try {
      r["canonical"] = canonical_policy(n);
    } catch (const std::exception& e) {
      r["canonical_error"] = std::string(e.what());
    }
    try {
      r["traits"] = describe_policy(policy_traits(n));
    } catch (const std::exception& e) {
      r["traits_error"] = std::string(e.what());
    }
    out[n.empty() ? std::string("<empty>") : n] = r;
  }
  return out;
}

std::vector<RunningGroup> random_running(CaseGen& g, int gpus) {
  std::vector<RunningGroup> run;
  int gpu = 0, id = 0;
  std::vector<int> order(gpus);
  for (int i = 0; i < gpus; ++i) order[i] = i;
  for (int i = gpus - 1; i > 0; --i) std::swap(order[i], order[g.below(i + 1)]);
  while (gpu < gpus) {
    const int w = std::min(gpus - gpu, g.pick({1, 1, 2, 2, 4, 8}));
    RunningGroup r;
    r.request_id = "r" + std::to_string(id++);
    for (int k = 0; k < w; ++k) r.group.push_back(order[gpu + k]);
    gpu += w;
    if (g.below(5) == 0) continue;  // idle GPUs
    r.stop_ms = g.pick({0.0, 20.0, 50.0, 80.0, 100.0, 120.0, 200.0});
    r.remaining_ms = g.pick({0.0, 40.0, 100.0, 300.0, 600.0, 1500.0, 4000.0});
    r.resume_ms = g.pick({0.0, 10.0, 25.0, 60.0});
    r.rung = g.below(4) == 0;
    run.push_back(r);
  }
  return run;
}

Json group_json(const std::vector<RunningGroup>& run) {
  Json a = Json::array();
  for (const auto& r : run) {
    Json o = Json::object();
    o["id"] = r.request_id;
    Json gg = Json::array();
    for (int x : r.group) gg.push_back(x);
    o["group"] = gg;
    o["stop"] = r.stop_ms;
    o["remaining"] = r.remaining_ms;
    o["resume"] = r.resume_ms;
    o["rung"] = r.rung;
    a.push_back(o);
  }
  return a;
}

Json preemption_decisions() {
  Json out = Json::object();
  Json groups = Json::array();
  CaseGen g(101);
  for (int c = 0; c < 300; ++c) {
    const int gpus = g.pick({2, 4, 4, 8, 8, 8, 16});
    auto run = random_running(g, gpus);
    std::vector<int> aff;
    const int n = 1 + g.below(6);
    for (int i = 0; i < n; ++i) aff.push_back(g.below(3) == 0 ? g.below(gpus) : -1);
    Json rec = Json::object();
    Json aj = Json::array();
    for (int a : aff) aj.push_back(a);
    rec["affinities"] = aj;
    rec["running"] = group_json(run);
    try {
      Json sel = Json::array();
      for (const auto& id : select_preemption_groups(aff, run)) sel.push_back(id);
      rec["selected"] = sel;
    } catch (const std::exception& e) {
      rec["error"] = std::string(e.what());
    }
    groups.push_back(rec);
  }
  out["groups"] = groups;
  Json deadline = Json::array();
  CaseGen h(202);
  for (int c = 0; c < 400; ++c) {
    const int gpus = h.pick({2, 4, 8, 8, 16});
    auto run = random_running(h, gpus);
    const double now = h.pick({0.0, 100.0, 1000.0});
    std::vector<ImageDemand> dem;
    const int n = 1 + h.below(5);
    for (int i = 0; i < n; ++i) {
      ImageDemand d;
      d.affinity = h.below(4) == 0 ? h.below(gpus) : -1;
      d.service_ms = h.pick({100.0, 300.0, 400.0, 1000.0});
      d.deadline_ms = now + d.service_ms * h.pick({0.5, 0.85, 0.9, 1.0, 1.2, 1.35, 1.4, 2.0, 4.0}) +
                      h.pick({0.0, 0.0, 20.0, 120.0});
      dem.push_back(d);
    }
    Json rec = Json::object();
    rec["now"] = now;
    Json dj = Json::array();
    for (const auto& d : dem) {
      Json o = Json::object();
      o["affinity"] = d.affinity;
      o["deadline"] = d.deadline_ms;
      o["service"] = d.service_ms;
      dj.push_back(o);
    }
    rec["waiting"] = dj;
    rec["running"] = group_json(run);
    try {
      auto r = select_deadline_preemption(now, dem, run);
      Json sel = Json::array();
      for (const auto& id : r.selected) sel.push_back(id);
      rec["selected"] = sel;
      rec["skips"] = static_cast<long long>(r.deadline_skips);
    } catch (const std::exception& e) {
      rec["error"] = std::string(e.what());
    }
    deadline.push_back(rec);
  }
  out["deadline"] = deadline;
  Json timing = Json::array();
  CaseGen t(303);
  for (int c = 0; c < 60; ++c) {
    const double block = t.pick({0.0, 5.0, 12.5, 40.0});
    const int total = t.pick({0, 30, 60});
    const int done = t.pick({-1, 0, 10, 30, 70});
    const double elapsed = t.pick({0.0, 3.0, 500.0});
    const int check = t.pick({0, 1, 2, 4});
    const int per = t.pick({1, 2});
    const bool delayed = t.below(2) == 0;
    Json rec = Json::object();
    rec["in"] = Json::parse("[" + std::to_string(block) + "," + std::to_string(total) + "," + std::to_string(done) +
                            "," + std::to_string(elapsed) + "," + std::to_string(check) + "," +
                            std::to_string(per) + "," + (delayed ? "true" : "false") + "]");
    try {
      auto e = estimate_preemption_timing(block, total, done, elapsed, check, per, delayed);
      rec["stop"] = e.stop_ms;
      rec["remaining"] = e.remaining_ms;
    } catch (const std::exception& e) {
      rec["error"] = std::string(e.what());
    }
    try {
      rec["converts"] = preemption_converts_deadline(elapsed, block * 40 + elapsed, block * 10, block * check,
                                                     block * total - elapsed);
    } catch (const std::exception& e) {
      rec["converts_error"] = std::string(e.what());
    }
    timing.push_back(rec);
  }
  out["timing"] = timing;
  return out;
}

Json snapshot_json() {
  ClusterCost c(profile());
  Json out = Json::object();
  // 1. simulator outcome per policy on one seeded trace
  Json ph = Json::parse(R"({"generator":{"count":48,"seed":23,"pattern":"gamma","cv":2,"rate_rpm":150,
     "classes":[{"weight":2,"kind":"video","class":"vid","service_ms":8000,"slo_scale_range":[1.1,2]},
                {"weight":2,"kind":"image","class":"img","service_ms":400,"slo_scale_range":[1.1,2]},
                {"weight":1,"kind":"image","class":"big","service_ms":1300,"slo_scale_range":[1.1,2]}]}})");
  const Json rows = study_workload(ph);
  Json sims = Json::object();
  const Json catalog = policy_catalog();
  for (const auto& p : catalog.as_array()) {
    const std::string id = p.at("id").as_string();
    auto r = simulate_cluster(rows, 8, id, c);
    Json s = Json::object();
    s["completed"] = r.summary.at("completed");
    s["slo_attainment"] = round6(r.summary.at("slo_attainment").as_double());
    for (const char* k : {"quanta", "plans", "preemptions", "resizes", "batches"})
      if (r.counters.contains(k)) s[k] = r.counters.at(k);
    sims[id] = s;
  }
  out["simulate"] = sims;
  // 2. planner assignments on fixed states
  Json states = Json::parse(R"([
    {"now_ms":0,"gpus":8,"busy":[false,false,false,false,false,false,false,false],"requests":[
      {"request_id":"v0","kind":"video","class":"vid","arrival_ms":0,"deadline_ms":1500,"steps_done":0},
      {"request_id":"v1","kind":"video","class":"vid","arrival_ms":0,"deadline_ms":5000,"steps_done":0},
      {"request_id":"v2","kind":"video","class":"vid","arrival_ms":0,"deadline_ms":5001,"steps_done":0},
      {"request_id":"i0","kind":"image","class":"img","arrival_ms":0,"deadline_ms":900},
      {"request_id":"i1","kind":"image","class":"big","arrival_ms":0,"deadline_ms":4000}]},
    {"now_ms":100,"gpus":4,"busy":[true,false,false,false],"requests":[
      {"request_id":"m","kind":"video","class":"vid","arrival_ms":0,"deadline_ms":9000,"status":"suspended",
       "steps_done":4,"blocks_done":12,"group":[2,3],"form":"cfg2"},
      {"request_id":"b","kind":"video","class":"vid","arrival_ms":0,"deadline_ms":8000,"status":"suspended",
       "steps_done":3,"blocks_done":0,"group":[0,1],"form":"cfg2"},
      {"request_id":"i","kind":"image","class":"img","arrival_ms":50,"deadline_ms":2000}]},
    {"now_ms":0,"gpus":2,"busy":[false,false],"requests":[
      {"request_id":"a","kind":"image","class":"img","arrival_ms":0,"deadline_ms":3000},
      {"request_id":"b","kind":"image","class":"img","arrival_ms":0,"deadline_ms":3000},
      {"request_id":"c","kind":"image","class":"big","arrival_ms":0,"deadline_ms":9000},
      {"request_id":"d","kind":"video","class":"vid","arrival_ms":0,"deadline_ms":1e9,"steps_done":10}]}
  ])");
  Json plans = Json::object();
  for (const char* pol : {"ditserve", "ditserve-b200", "ditserve-v1", "tetriserve", "sbp-esp-cfg2", "edf-bestfit",
                          "xdit-sp1", "partition", "abl-no-cb", "block-cfg2"}) {
    Json per = Json::array();
    for (const auto& st : states.as_array()) per.push_back(cluster_plan(st, pol, c));
    plans[pol] = per;
  }
  out["plan"] = plans;
  // 3. online selector decisions on fixed queues
  Json q = Json::parse(R"([
    {"request_id":"v","kind":"video","arrival_ms":0,"deadline_ms":60000,"remaining_ms":30000,"service_ms":30000,
     "ready_since_ms":0,"action":"denoise","started":true,"ready":true,"release_ms":0,"stage_deadline_ms":60000,
     "remaining_total_ms":30000,"action_ms_by_quantum":{"1":600,"2":1200,"4":2400,"8":4800,"step":600}},
    {"request_id":"i","kind":"image","arrival_ms":1000,"deadline_ms":3000,"remaining_ms":400,"service_ms":400,
     "ready_since_ms":1000,"action":"image","started":false,"ready":true,"release_ms":1000,"stage_deadline_ms":3000,
     "remaining_total_ms":400,"action_ms_by_quantum":{"1":400,"2":800,"4":1600,"8":3200,"step":400}}])");
  Json online = Json::object();
  for (const char* pol : {"fcfs", "edf", "srtf", "session_serial", "stage_edf", "session_slack", "edf_b1", "edf_b4",
                          "edf_step", "guarded_b4", "guarded_adaptive", "feasible_b4"})
    if (is_online_policy(pol))
      online[pol] = select_online(q, 1200, pol, "v", Json(1), Json::parse(R"({"image_deadline_ms": 2000})"));
  out["online"] = online;
  // 4. policy-name resolution and 5. block-preemption selection on generated cases
  out["names"] = name_resolution();
  out["preemption"] = preemption_decisions();
  return out;
}

}  // namespace

TEST("decisions match the golden fixture") {
  const std::string path = std::string(DS_FIXTURE_DIR) + "/control-golden.json";
  const Json now = snapshot_json();
  if (const char* up = std::getenv("DS_UPDATE_GOLDEN"); up && std::string(up) == "1") {
    std::ofstream(path) << now.dump(1) << "\n";
    std::cout << "  fixture rewritten: " << path << "\n";
    return;
  }
  std::ifstream f(path);
  CHECK(static_cast<bool>(f));
  if (!f) return;
  std::stringstream ss;
  ss << f.rdbuf();
  const Json want = Json::parse(ss.str());
  for (const char* part : {"simulate", "plan", "online", "names", "preemption"}) {
    for (const auto& [k, v] : want.at(part).as_object()) {
      const bool same = now.at(part).contains(k) && now.at(part).at(k) == v;
      if (!same) std::cerr << "  golden diff in " << part << "/" << k << "\n    want " << v.dump() << "\n    got  "
                           << (now.at(part).contains(k) ? now.at(part).at(k).dump() : std::string("<missing>")) << "\n";
      CHECK(same);
    }
    CHECK(now.at(part).size() == want.at(part).size());
  }
}

TEST("the golden snapshot is deterministic within a process") {
  CHECK(snapshot_json() == snapshot_json());
}

int main() { return dstest::run_all(); }
