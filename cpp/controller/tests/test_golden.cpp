// Golden decision fixture: the simulator's outcome for every registered policy on a seeded
// mixed trace, the planner's assignments on a set of fixed cluster states, and the online
// selector's decisions on fixed queues, compared against tests/fixtures/control-golden.json.
// Any change of a decision rule shows up here as a diff; after an intended change, rebuild
// the fixture with DS_UPDATE_GOLDEN=1 and review the diff.  (The reference keeps such a
// fixture for its control rules: tests/fixtures/control-baseline.json.)
#include <cmath>
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
  for (const char* part : {"simulate", "plan", "online"}) {
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
