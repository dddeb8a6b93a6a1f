// Planner, preemption selectors and simulator scenarios (one behaviour per check).
#include <set>

#include "check.hpp"
#include "ds/planner.hpp"
#include "ds/sim.hpp"
#include "ds/study.hpp"
#include "ds/workload.hpp"

using namespace ds;

namespace {

Json profile() {
  return Json::parse(R"({"links":{"default_gbps":700,"default_latency_ms":0.02},
   "sp_efficiency":{"2":0.97,"4":0.94,"8":0.88},"quantum_overhead_ms":0,"resize_ms":0,
   "classes":{
    "vid":{"kind":"video","steps":10,"blocks_per_step":30,"heads":12,"step_compute_ms":800,
           "comm_mb_per_step":20000,"collectives_per_step":240,"cfg_exchange_mb":4,"decode_ms":100,"decode_chunks":1},
    "img":{"kind":"image","steps":28,"tokens":1024,"step_ms":12,"service_ms":400,"decode_ms":50,
           "batch_step_ms":{"1":12,"2":16,"4":26,"8":46}},
    "big":{"kind":"image","steps":28,"tokens":4096,"step_ms":40,"service_ms":1300,"decode_ms":180,
           "batch_step_ms":{"1":40,"2":74,"4":142,"8":280}}}})");
}

Json req(const std::string& id, const std::string& kind, const std::string& klass, double arrival, double deadline,
         int steps_done = 0) {
  Json r = Json::object();
  r["request_id"] = id;
  r["kind"] = kind;
  r["class"] = klass;
  r["arrival_ms"] = arrival;
  r["deadline_ms"] = deadline;
  r["status"] = "waiting";
  if (kind == "video") r["steps_done"] = steps_done;
  return r;
}

Json state(int gpus, std::vector<Json> reqs, std::vector<int> busy = {}, double now = 0) {
  Json s = Json::object();
  s["now_ms"] = now;
  s["gpus"] = gpus;
  Json b = Json::array();
  for (int i = 0; i < gpus; ++i) b.push_back(std::count(busy.begin(), busy.end(), i) > 0);
  s["busy"] = b;
  Json r = Json::array();
  for (auto& x : reqs) r.push_back(x);
  s["requests"] = r;
  return s;
}

const Json* find(const Json& plan, const std::string& id) {
  for (const auto& a : plan.at("assignments").as_array())
    if (a.at("request_id").as_string() == id) return &a;
  return nullptr;
}

}  // namespace

TEST("aligned groups are contiguous") {
  auto g = cluster_groups(8, 4);
  CHECK(g.size() == 2 && g[1][0] == 4 && g[1][3] == 7);
  CHECK(cluster_groups(8, 3).size() == 2);
}

TEST("static form places every video on its fixed form") {
  ClusterCost c(profile());
  auto p = cluster_plan(state(8, {req("a", "video", "vid", 0, 1e9), req("b", "video", "vid", 0, 1e9)}),
                        "static-cfg2sp2", c);
  CHECK(find(p, "a") && find(p, "a")->at("form").as_string() == "cfg2sp2");
  CHECK(find(p, "b") && find(p, "b")->at("degree").as_int() == 4);
  std::set<long long> used;
  for (const auto& a : p.at("assignments").as_array())
    for (const auto& g : a.at("group").as_array()) CHECK(used.insert(g.as_int()).second);
}

TEST("ditserve admits videos on at least a CFG pair and prunes dominated forms") {
  ClusterCost c(profile());
  auto forms = candidate_forms(policy_traits("ditserve"), c, "vid", 8, Json::object());
  for (const auto& f : forms) CHECK(f.degree() >= 2);
  // cfg2 (one exchange) beats sp2 (all-to-all) at two GPUs on NVSwitch
  CHECK(form_name(forms.front()) == "cfg2");
  auto p = cluster_plan(state(8, {req("a", "video", "vid", 0, 1e9)}), "ditserve", c);
  CHECK(find(p, "a")->at("degree").as_int() >= 2);
}

TEST("feasible minimal form meets the deadline") {
  ClusterCost c(profile());
  // 10 steps x 800 ms = 8 s on one GPU; deadline 3 s needs >= 4 GPUs
  auto p = cluster_plan(state(8, {req("a", "video", "vid", 0, 3000)}), "abl-step-elastic", c);
  const Json* a = find(p, "a");
  CHECK(a != nullptr);
  CHECK(a->at("degree").as_int() >= 4);
  CHECK(c.remaining_ms(req("a", "video", "vid", 0, 3000), parse_form(a->at("form").as_string())) <= 3000);
}

TEST("late requests are demoted behind feasible ones") {
  ClusterCost c(profile());
  auto late = req("late", "video", "vid", 0, 10);      // impossible
  auto ok = req("ok", "video", "vid", 5, 20000);
  auto p = cluster_plan(state(1, {late, ok}), "abl-step-elastic", c);
  CHECK(find(p, "ok") != nullptr);
  CHECK(find(p, "late") == nullptr);
  // EDF-BF does not demote: the earliest deadline goes first even when late
  auto q = cluster_plan(state(1, {late, ok}), "edf-bestfit", c);
  CHECK(find(q, "late") != nullptr);
}

TEST("srtf and fcfs orders") {
  ClusterCost c(profile());
  auto a = req("long", "video", "vid", 0, 1e9, 0);
  auto b = req("short", "video", "vid", 1, 1e9, 9);
  Json o = Json::object();
  o["order"] = "srtf";
  auto p = cluster_plan(state(1, {a, b}), "abl-step-elastic", c, o);
  CHECK(find(p, "short") != nullptr && find(p, "long") == nullptr);
  o["order"] = "fcfs";
  p = cluster_plan(state(1, {a, b}), "abl-step-elastic", c, o);
  CHECK(find(p, "long") != nullptr);
}

TEST("pair_fit keeps free pairs whole for videos") {
  ClusterCost c(profile());
  // GPU 0 busy: an image should take GPU 1 (partner busy) rather than break pair 2-3
  auto p = cluster_plan(state(4, {req("i", "image", "img", 0, 1e9)}, {0}), "ditserve", c);
  CHECK(find(p, "i")->at("group")[0].as_int() == 1);
  auto q = cluster_plan(state(4, {req("i", "image", "img", 0, 1e9)}, {0}), "abl-first-fit", c);
  CHECK(find(q, "i")->at("group")[0].as_int() == 1);
  auto r = cluster_plan(state(4, {req("i", "image", "img", 0, 1e9)}, {2}), "ditserve", c);
  CHECK(find(r, "i")->at("group")[0].as_int() == 3);
}

TEST("feasible images are boosted ahead of videos in the full system") {
  ClusterCost c(profile());
  auto v = req("v", "video", "vid", 0, 5000);
  auto i = req("i", "image", "img", 0, 6000);
  auto p = cluster_plan(state(2, {v, i}), "ditserve", c);
  CHECK(find(p, "i") != nullptr);
  auto q = cluster_plan(state(2, {v, i}), "abl-no-img-priority", c);
  CHECK(find(q, "v") != nullptr);
}

TEST("continuous batching groups images that keep their deadlines") {
  ClusterCost c(profile());
  std::vector<Json> rs;
  for (int k = 0; k < 5; ++k) rs.push_back(req("i" + std::to_string(k), "image", "img", 0, 5000));
  auto p = cluster_plan(state(1, rs), "ditserve", c);
  CHECK(p.at("assignments").size() == 1);
  const Json& a = p.at("assignments")[0];
  CHECK(a.at("quantum").as_string() == "continuous_batch");
  CHECK(a.at("batch").size() == 5);
  // a tight deadline member is not joined into a batch that would make it late
  std::vector<Json> rs2 = {req("x", "image", "img", 0, 5000), req("y", "image", "img", 0, 5000)};
  rs2[1]["deadline_ms"] = 12 * 28 + 50 + 1.0;  // exactly fits alone
  auto q = cluster_plan(state(1, rs2), "ditserve", c);
  CHECK(q.at("assignments")[0].get("batch").size() <= 2);
  auto nb = cluster_plan(state(1, rs), "abl-no-cb", c);
  CHECK(nb.at("assignments")[0].at("quantum").as_string() == "atomic");
}

TEST("deadline knapsack keeps the most requests on track") {
  ClusterCost c(profile());
  // 4 GPUs, three videos: two can be saved with 2 GPUs each, the third would need the whole node
  auto a = req("a", "video", "vid", 0, 5000);   // needs >= 2 GPUs
  auto b = req("b", "video", "vid", 0, 5000);
  auto x = req("x", "video", "vid", 0, 1500);   // needs 8 -> unsavable on 4
  auto p = cluster_plan(state(4, {x, a, b}), "tetriserve", c);
  CHECK(find(p, "a") && find(p, "b"));
  CHECK(find(p, "x") == nullptr);
}

TEST("EDF best fit redistributes surplus GPUs") {
  ClusterCost c(profile());
  auto a = req("a", "video", "vid", 0, 1e9);
  auto p = cluster_plan(state(8, {a}), "edf-bestfit", c);
  // 12 heads: the widest plain-Ulysses group is sp4 (sp8 does not divide the heads)
  CHECK(find(p, "a")->at("degree").as_int() == 4);
  auto q = cluster_plan(state(8, {a}), "edf-bestfit-cfg2", c);
  CHECK(find(q, "a")->at("degree").as_int() == 8);
}

TEST("round baselines hold GPUs for round_steps steps") {
  ClusterCost c(profile());
  auto p = cluster_plan(state(8, {req("a", "video", "vid", 0, 1e9)}), "tetriserve", c);
  CHECK(find(p, "a")->at("steps").as_int() == 5);
}

TEST("partition reserves an image share") {
  ClusterCost c(profile());
  std::vector<Json> vids;
  for (int k = 0; k < 4; ++k) vids.push_back(req("v" + std::to_string(k), "video", "vid", 0, 1e9));
  auto p = cluster_plan(state(8, vids), "partition", c);
  for (const auto& a : p.at("assignments").as_array())
    for (const auto& g : a.at("group").as_array()) CHECK(g.as_int() < 6);
}

TEST("decode shrinks to one GPU unless the policy holds the group") {
  ClusterCost c(profile());
  auto v = req("v", "video", "vid", 0, 1e9, 10);
  v["group"] = Json::parse("[0,1,2,3]");
  v["form"] = "sp4";
  v["status"] = "suspended";
  auto p = cluster_plan(state(8, {v}), "ditserve", c);
  CHECK(find(p, "v")->at("quantum").as_string() == "finish");
  CHECK(find(p, "v")->at("degree").as_int() == 1);
  auto q = cluster_plan(state(8, {v}), "abl-no-decode-shrink", c);
  CHECK(find(q, "v")->at("degree").as_int() == 4);
}

TEST("xdit baseline resumes a started request on its own GPUs") {
  ClusterCost c(profile());
  auto v = req("v", "video", "vid", 0, 1e9, 3);
  v["group"] = Json::parse("[2,3]");
  v["form"] = "sp2";
  v["status"] = "suspended";
  auto w = req("w", "video", "vid", 0, 10, 0);
  auto p = cluster_plan(state(8, {w, v}), "xdit-sp2", c);
  CHECK(find(p, "v")->at("group")[0].as_int() == 2);
}

TEST("block preemption rings a running video for a waiting tight image") {
  ClusterCost c(profile());
  auto v = req("v", "video", "vid", 0, 1e9, 2);
  v["status"] = "running";
  v["group"] = Json::parse("[0]");
  v["form"] = "sp1";
  v["quantum_started_ms"] = 0.0;
  auto i = req("i", "image", "img", 0, 800);  // 400 ms service, the video's step ends at 800 ms
  auto p = cluster_plan(state(1, {v, i}, {0}, 0), "ditserve", c);
  CHECK(p.at("preempt").size() == 1);
  auto q = cluster_plan(state(1, {v, i}, {0}, 0), "abl-no-block", c);
  CHECK(q.at("preempt").size() == 0);
}

TEST("preemption timing and deadline conversion") {
  auto t = estimate_preemption_timing(10, 30, 5, 20, 2, 1, true);
  CHECK_NEAR(t.stop_ms, 40.0, 1e-12);
  CHECK_NEAR(t.remaining_ms, 230.0, 1e-12);
  CHECK(preemption_converts_deadline(0, 100, 50, 40, 200));
  CHECK(!preemption_converts_deadline(0, 300, 50, 40, 200));  // on time anyway
  CHECK(!preemption_converts_deadline(0, 60, 50, 40, 200));   // late either way
  CHECK_THROWS(estimate_preemption_timing(0, 30, 0, 0, 1, 1, false));
}

TEST("min-cost preemption selection frees enough GPUs") {
  std::vector<RunningGroup> run = {{"a", {0, 1}, 10, 100, 0, false}, {"b", {2}, 50, 100, 0, false},
                                   {"c", {3}, 5, 100, 0, false}};
  auto s = select_preemption_groups({-1}, run);
  CHECK(s.size() == 1 && s[0] == "c");
  auto s2 = select_preemption_groups({2}, run);  // pinned to GPU 2
  CHECK(std::find(s2.begin(), s2.end(), "b") != s2.end());
  CHECK_THROWS(select_preemption_groups({-1}, {{"a", {0}, 1, 1, 0, false}, {"b", {0}, 1, 1, 0, false}}));
}

TEST("deadline preemption only rings groups that save their image") {
  std::vector<RunningGroup> run = {{"v", {0}, 30, 900, 0, false}};
  auto s = select_deadline_preemption(0, {{-1, 500, 400}}, run);
  CHECK(s.selected.size() == 1);
  auto s2 = select_deadline_preemption(0, {{-1, 5000, 400}}, run);  // patient finish is on time
  CHECK(s2.selected.empty());
  auto s3 = select_deadline_preemption(0, {{-1, 100, 400}}, run);   // hopeless
  CHECK(s3.selected.empty() && s3.deadline_skips == 1);
}

TEST("plan trace is bounded and decision-free") {
  ClusterCost c(profile());
  std::vector<Json> rs;
  for (int k = 0; k < 100; ++k) rs.push_back(req("i" + std::to_string(k), "image", "img", 0, 1e9));
  PlanTrace tr;
  auto with = cluster_plan(state(8, rs), "ditserve", c, Json::object(), &tr);
  auto without = cluster_plan(state(8, rs), "ditserve", c);
  CHECK(with == without);
  CHECK(tr.rows.size() == 64 && tr.dropped == 36);
}

TEST("simulator replays a mixed trace for every registered policy") {
  ClusterCost c(profile());
  Json ph = Json::parse(R"({"generator":{"count":40,"seed":11,"pattern":"poisson","rate_rpm":30,
     "classes":[{"weight":2,"kind":"video","class":"vid","service_ms":8000,"slo_scale_range":[1.5,3]},
                {"weight":1,"kind":"image","class":"img","service_ms":400,"slo_scale_range":[1.5,3]},
                {"weight":1,"kind":"image","class":"big","service_ms":1300,"slo_scale_range":[1.5,3]}]}})");
  Json rows = study_workload(ph);
  double best = 0, base = 1;
  for (const char* pol : {"ditserve", "tetriserve", "sbp-esp", "edf-bestfit", "static-cfg2sp4", "xdit-sp1",
                          "abl-no-block", "cfg2-first", "partition", "ditserve-v1", "stair-base"}) {
    auto r = simulate_cluster(rows, 8, pol, c);
    CHECK(r.summary.at("requests").as_int() == 40);
    CHECK(r.summary.at("completed").as_int() == 40);
    const double sar = r.summary.at("slo_attainment").as_double();
    if (std::string(pol) == "ditserve") best = sar;
    if (std::string(pol) == "xdit-sp1") base = sar;
  }
  CHECK(best >= base);
}

TEST("simulator is deterministic and uses the planner profile for decisions") {
  ClusterCost c(profile());
  Json ph = Json::parse(R"({"generator":{"count":20,"seed":5,"pattern":"gamma","rate_rpm":20,"cv":2,
     "classes":[{"kind":"video","class":"vid","service_ms":8000,"slo_scale":2},
                {"kind":"image","class":"img","service_ms":400,"slo_scale":2}]}})");
  Json rows = study_workload(ph);
  auto a = simulate_cluster(rows, 8, "ditserve", c);
  auto b = simulate_cluster(rows, 8, "ditserve", c);
  CHECK(a.rows == b.rows);
  Json wrong = profile();
  wrong["classes"]["vid"]["step_compute_ms"] = 8000;
  ClusterCost w(wrong);
  auto d = simulate_cluster(rows, 8, "ditserve", c, Json::object(), &w);
  CHECK(d.summary.at("completed").as_int() == 20);
}

int main() { return dstest::run_all(); }
