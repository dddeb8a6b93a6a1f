// Planner, cost-model and simulator scenarios beyond the basic planner checks: solver-step
// ownership, class memory minimums, pairs, atomic image batches, chunked decode quanta,
// contention and overhead terms, pruning on slow links, widening, aliases and simulation
// accounting.  One behaviour per check.
#include <algorithm>
#include <set>

#include "check.hpp"
#include "ds/planner.hpp"
#include "ds/policy.hpp"
#include "ds/sim.hpp"
#include "ds/study.hpp"
#include "ds/workload.hpp"

using namespace ds;

namespace {

Json profile(double gbps = 700) {
  Json p = Json::parse(R"({"links":{"default_latency_ms":0.02},
   "sp_efficiency":{"2":0.97,"4":0.94,"8":0.88},"quantum_overhead_ms":0,"resize_ms":0,
   "classes":{
    "vid":{"kind":"video","steps":10,"blocks_per_step":30,"heads":12,"step_compute_ms":800,
           "comm_mb_per_step":20000,"collectives_per_step":240,"cfg_exchange_mb":4,"decode_ms":100,"decode_chunks":1},
    "long":{"kind":"video","steps":10,"blocks_per_step":30,"heads":24,"step_compute_ms":800,
           "comm_mb_per_step":20000,"collectives_per_step":240,"cfg_exchange_mb":4,"decode_ms":400,"decode_chunks":4},
    "img":{"kind":"image","steps":28,"tokens":1024,"step_ms":12,"service_ms":400,"decode_ms":50,
           "batch_ms":{"1":400,"2":520,"4":800},
           "batch_step_ms":{"1":12,"2":16,"4":26,"8":46}}}})");
  p["links"]["default_gbps"] = gbps;
  return p;
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

Json suspended(const std::string& id, const char* group, const char* form, int steps_done, int blocks_done) {
  Json v = req(id, "video", "vid", 0, 1e9, steps_done);
  v["status"] = "suspended";
  v["group"] = Json::parse(group);
  v["form"] = form;
  v["blocks_done"] = blocks_done;
  return v;
}

}  // namespace

TEST("a request inside a solver step resumes on its own group and form") {
  ClusterCost c(profile());
  auto v = suspended("v", "[2,3]", "cfg2", 3, 12);
  auto p = cluster_plan(state(8, {v}), "ditserve", c);
  const Json* a = find(p, "v");
  CHECK(a != nullptr);
  CHECK(a->at("group")[0].as_int() == 2 && a->at("group")[1].as_int() == 3);
  CHECK(a->at("form").as_string() == "cfg2");
  CHECK(a->at("reason").as_string() == "mid-step");
}

TEST("the plan never moves a mid-step request onto other GPUs") {
  ClusterCost c(profile());
  auto v = suspended("v", "[2,3]", "cfg2", 3, 12);
  auto p = cluster_plan(state(8, {v}, {3}), "ditserve", c);  // GPU 3 busy: wait, do not move
  CHECK(find(p, "v") == nullptr);
  auto b = suspended("b", "[2,3]", "cfg2", 3, 0);            // at a step boundary: free to move
  auto q = cluster_plan(state(8, {b}, {3}), "ditserve", c);
  CHECK(find(q, "b") != nullptr);
}

TEST("classes that do not fit one GPU get their minimum degree") {
  Json pr = profile();
  pr["classes"]["vid"]["min_degree"] = 4;
  ClusterCost c(pr);
  for (const char* pol : {"abl-step-elastic", "edf-bestfit", "ditserve"}) {
    auto forms = candidate_forms(policy_traits(pol), c, "vid", 8, Json::object());
    CHECK(!forms.empty());
    for (const auto& f : forms) CHECK(f.degree() >= 4);
  }
  auto p = cluster_plan(state(8, {req("a", "video", "vid", 0, 1e9)}, {0, 1, 2, 3, 4}), "abl-step-elastic", c);
  CHECK(find(p, "a") == nullptr);  // three free GPUs are not enough
}

TEST("heads divisibility removes Ulysses forms that do not split the heads") {
  ClusterCost c(profile());
  auto forms = candidate_forms(policy_traits("abl-step-elastic"), c, "vid", 8, Json::object());
  for (const auto& f : forms) CHECK(12 % f.ulysses() == 0);
  auto wide = candidate_forms(policy_traits("abl-step-elastic"), c, "long", 8, Json::object());
  bool has8 = false;
  for (const auto& f : wide) has8 = has8 || f.degree() == 8;
  CHECK(has8);
}

TEST("lockstep pairing joins a second video onto a placed group") {
  Json pr = profile();
  pr["pair_overlap"] = 0.5;
  ClusterCost c(pr);
  Json o = Json::object();
  o["pairing"] = true;
  o["forms"] = Json::parse(R"(["sp2"])");  // an SP form: one request's all-to-all hides under the other's compute
  auto a = req("a", "video", "vid", 0, 1e9);
  auto b = req("b", "video", "vid", 1, 1e9);
  auto p = cluster_plan(state(2, {a, b}), "ditserve", c, o);
  const Json* pa = find(p, "a");
  const Json* pb = find(p, "b");
  CHECK(pa && pb);
  CHECK(pa->at("pair").as_string() == "b" && pb->at("pair").as_string() == "a");
  CHECK(pa->at("group") == pb->at("group"));
  o["pairing"] = false;
  auto q = cluster_plan(state(2, {a, b}), "ditserve", c, o);
  CHECK(find(q, "b") == nullptr);
  CHECK(c.pair_ms("vid", "vid", parse_form("cfg2")) >= 2 * c.step_ms("vid", parse_form("cfg2")) - 1e-9);
}

TEST("atomic image batches for batching baselines") {
  ClusterCost c(profile());
  std::vector<Json> rs;
  for (int k = 0; k < 3; ++k) rs.push_back(req("i" + std::to_string(k), "image", "img", 0, 1e9));
  auto p = cluster_plan(state(1, rs), "sbp-esp", c);
  CHECK(p.at("assignments").size() == 1);
  const Json& a = p.at("assignments")[0];
  CHECK(a.at("quantum").as_string() == "atomic");
  CHECK(a.at("batch").size() == 3);
  CHECK(a.at("reason").as_string() == "image-batch");
}

TEST("chunked decode is preemptible between latent frames") {
  ClusterCost c(profile());
  Json v = req("v", "video", "long", 0, 1e9, 10);
  v["status"] = "suspended";
  v["group"] = Json::parse("[0,1]");
  v["form"] = "cfg2";
  v["decode_done"] = 1;
  auto p = cluster_plan(state(8, {v}), "ditserve", c);
  CHECK(find(p, "v")->at("quantum").as_string() == "finish");
  CHECK(find(p, "v")->at("decode_frames").as_int() == 1);  // block policies: one chunk per quantum
  auto q = cluster_plan(state(8, {v}), "abl-step-elastic", c);
  CHECK(find(q, "v")->at("decode_frames").as_int() == 3);  // the rest in one go
  CHECK_NEAR(c.chunk_ms("long"), 100.0, 1e-9);
}

TEST("per-block overhead is charged once per block") {
  Json pr = profile();
  pr["block_overhead_ms"] = 0.5;
  ClusterCost c(pr);
  ClusterCost z(profile());
  const Form f = parse_form("sp2");
  CHECK_NEAR(c.block_ms("vid", f) - z.block_ms("vid", f), 0.5, 1e-9);
  CHECK_NEAR(c.block_ms("vid", parse_form("cfg2")) - z.block_ms("vid", parse_form("cfg2")), 0.25, 1e-9);
}

TEST("concurrent SP groups see the contention table") {
  Json pr = profile();
  pr["links"]["2"] = Json::parse(R"({"gbps":700,"concurrent_gbps":{"1":700,"4":350}})");
  ClusterCost c(pr);
  const Form f = parse_form("sp2");
  CHECK(c.step_ms("vid", f, 4) > c.step_ms("vid", f, 1));
  CHECK_NEAR(c.step_ms("vid", f, 1), ClusterCost(profile()).step_ms("vid", f, 1), 1e-9);
}

TEST("measured form entries override the formula and stay per class") {
  Json pr = profile();
  pr["classes"]["vid"]["forms"] = Json::parse(R"({"cfg2":{"step_ms":123.0}})");
  ClusterCost c(pr);
  CHECK_NEAR(c.step_ms("vid", parse_form("cfg2")), 123.0, 1e-12);
  CHECK(c.terms("vid", parse_form("cfg2")).measured);
  CHECK(!c.terms("long", parse_form("cfg2")).measured);
}

TEST("slow links make wide Ulysses forms dominated and pruned") {
  ClusterCost slow(profile(2.0));  // 2 GB/s: the all-to-all dominates
  auto forms = candidate_forms(policy_traits("ditserve"), slow, "vid", 8, Json::object());
  for (const auto& f : forms) CHECK(f.sp == 1);  // only CFG forms survive
  ClusterCost fast(profile(700));
  auto wide = candidate_forms(policy_traits("ditserve"), fast, "vid", 8, Json::object());
  bool has_sp = false;
  for (const auto& f : wide) has_sp = has_sp || f.sp > 1;
  CHECK(has_sp);
}

TEST("CFG-pair admission waits instead of starting narrow") {
  ClusterCost c(profile());
  auto p = cluster_plan(state(4, {req("a", "video", "vid", 0, 1e9)}, {0, 1, 2}), "ditserve", c);
  CHECK(find(p, "a") == nullptr);  // one free GPU: ditserve does not start at sp1
  auto q = cluster_plan(state(4, {req("a", "video", "vid", 0, 1e9)}, {0, 1, 2}), "stair-base", c);
  CHECK(find(q, "a") != nullptr && find(q, "a")->at("degree").as_int() == 1);
}

TEST("a lone video is widened while scaling stays efficient") {
  ClusterCost c(profile());
  auto p = cluster_plan(state(8, {req("a", "video", "vid", 0, 1e9)}), "ditserve", c);
  CHECK(find(p, "a")->at("degree").as_int() == 8);
  CHECK(find(p, "a")->at("reason").as_string() == "widened");
  Json o = Json::object();
  o["widen_efficiency"] = 0.999;  // no form is that efficient: stay at the minimal one
  o["idle_widening"] = false;
  auto q = cluster_plan(state(8, {req("a", "video", "vid", 0, 1e9)}), "ditserve", c, o);
  CHECK(find(q, "a")->at("degree").as_int() == 2);
  // with idle widening the GPUs nobody else needs still go to the lone video
  o["idle_widening"] = true;
  auto w = cluster_plan(state(8, {req("a", "video", "vid", 0, 1e9)}), "ditserve", c, o);
  CHECK(find(w, "a")->at("degree").as_int() == 8);
  CHECK(find(w, "a")->at("reason").as_string() == "idle-widened");
}

TEST("widening stops while an image waits unplaced") {
  ClusterCost c(profile());
  std::vector<Json> rs = {req("a", "video", "vid", 0, 1e9)};
  for (int k = 0; k < 8; ++k) rs.push_back(req("i" + std::to_string(k), "image", "img", 0, 1e9));
  Json o = Json::object();
  o["continuous_batch"] = 1;  // one image per GPU: images saturate the node
  auto p = cluster_plan(state(8, rs), "ditserve", c, o);
  const Json* a = find(p, "a");
  CHECK(a == nullptr || a->at("degree").as_int() <= 2);
}

TEST("doorbell option off disables sub-step preemption") {
  ClusterCost c(profile());
  auto v = req("v", "video", "vid", 0, 1e9, 2);
  v["status"] = "running";
  v["group"] = Json::parse("[0]");
  v["form"] = "sp1";
  v["quantum_started_ms"] = 0.0;
  auto i = req("i", "image", "img", 0, 800);
  Json o = Json::object();
  o["doorbell"] = false;
  CHECK(cluster_plan(state(1, {v, i}, {0}), "ditserve", c).at("preempt").size() == 1);
  CHECK(cluster_plan(state(1, {v, i}, {0}), "ditserve", c, o).at("preempt").size() == 0);
}

TEST("block quanta are emitted only by block policies") {
  ClusterCost c(profile());
  Json o = Json::object();
  o["quantum_blocks"] = 6;
  auto p = cluster_plan(state(8, {req("a", "video", "vid", 0, 1e9)}), "ditserve", c, o);
  CHECK(find(p, "a")->at("quantum").as_int() == 6);
  auto q = cluster_plan(state(8, {req("a", "video", "vid", 0, 1e9)}), "abl-step-elastic", c, o);
  CHECK(find(q, "a")->at("quantum").as_string() == "step");
}

TEST("a started image keeps its GPU affinity") {
  ClusterCost c(profile());
  auto i = req("i", "image", "img", 0, 1e9);
  i["affinity"] = 5;
  auto p = cluster_plan(state(8, {i}), "ditserve", c);
  CHECK(find(p, "i")->at("group")[0].as_int() == 5);
  auto q = cluster_plan(state(8, {i}, {5}), "ditserve", c);
  CHECK(find(q, "i") == nullptr);
}

TEST("invalid planner input is rejected") {
  ClusterCost c(profile());
  CHECK_THROWS(cluster_plan(state(2, {req("a", "video", "vid", 0, 1), req("a", "image", "img", 0, 1)}), "ditserve", c));
  CHECK_THROWS(cluster_plan(state(2, {req("a", "audio", "img", 0, 1)}), "ditserve", c));
  Json s = state(2, {});
  s["busy"] = Json::parse("[false]");
  CHECK_THROWS(cluster_plan(s, "ditserve", c));
  Json o = Json::object();
  o["order"] = "lifo";
  CHECK_THROWS(cluster_plan(state(2, {}), "ditserve", c, o));
  o = Json::object();
  o["continuous_batch"] = 9;
  CHECK_THROWS(cluster_plan(state(2, {}), "ditserve", c, o));
}

TEST("legacy aliases plan as their canonical policy and retired names are refused") {
  ClusterCost c(profile());
  CHECK(canonical_policy("knapsack_dp") == "ditserve-v1");
  CHECK(canonical_policy("static_cfg2sp2") == "static-cfg2sp2");
  auto a = cluster_plan(state(8, {req("a", "video", "vid", 0, 1e9)}), "knapsack_dp", c);
  auto b = cluster_plan(state(8, {req("a", "video", "vid", 0, 1e9)}), "ditserve-v1", c);
  CHECK(a == b);
  CHECK_THROWS(policy_traits("vllm_omni"));
  CHECK_THROWS(policy_traits("no-such-policy"));
}

TEST("simulation accounting: every request is counted once and finishes after it starts") {
  ClusterCost c(profile());
  Json ph = Json::parse(R"({"generator":{"count":30,"seed":3,"pattern":"poisson","rate_rpm":40,
     "classes":[{"weight":1,"kind":"video","class":"vid","service_ms":8000,"slo_scale":2},
                {"weight":2,"kind":"image","class":"img","service_ms":400,"slo_scale":2}]}})");
  Json rows = study_workload(ph);
  auto r = simulate_cluster(rows, 4, "ditserve", c);
  CHECK(r.rows.size() == 30);
  int on_time = 0;
  for (const auto& row : r.rows.as_array()) {
    CHECK(row.at("status").as_string() == "done");
    CHECK(row.at("finish_ms").as_double() >= row.at("start_ms").as_double());
    CHECK(row.at("start_ms").as_double() >= row.at("arrival_ms").as_double());
    on_time += row.at("finish_ms").as_double() <= row.at("deadline_ms").as_double();
  }
  CHECK(r.summary.at("on_time").as_int() == on_time);
  CHECK(r.counters.at("quanta").as_int() >= 30);
}

TEST("a horizon censors unfinished requests") {
  ClusterCost c(profile());
  Json ph = Json::parse(R"({"generator":{"count":10,"seed":1,"pattern":"offline_all",
     "classes":[{"kind":"video","class":"vid","service_ms":8000,"slo_scale":2}]}})");
  auto r = simulate_cluster(study_workload(ph), 2, "ditserve", c, Json::object(), nullptr, 5000);
  CHECK(r.summary.at("completed").as_int() < 10);
  CHECK(r.summary.at("censored").as_int() + r.summary.at("completed").as_int() +
            r.summary.at("not_executed").as_int() == 10);
}

TEST("block preemption shortens image latency behind a long video on one GPU") {
  ClusterCost c(profile());
  Json rows = Json::parse(R"([
    {"request_id":"v","kind":"video","class":"vid","arrival_ms":0,"deadline_ms":1e9,"spec":{"steps":10}},
    {"request_id":"i","kind":"image","class":"img","arrival_ms":100,"deadline_ms":1100,"spec":{"steps":28}}])");
  auto with = simulate_cluster(rows, 1, "ditserve", c);
  auto without = simulate_cluster(rows, 1, "abl-no-block", c);
  auto fin = [](const SimResult& r, const std::string& id) {
    for (const auto& row : r.rows.as_array())
      if (row.at("request_id").as_string() == id) return row.at("finish_ms").as_double();
    return -1.0;
  };
  CHECK(fin(with, "i") < fin(without, "i"));
  CHECK(fin(with, "i") <= 1100);
}

TEST("elastic SP finishes a lone video sooner than a fixed single GPU") {
  ClusterCost c(profile());
  Json rows = Json::parse(R"([
    {"request_id":"v","kind":"video","class":"vid","arrival_ms":0,"deadline_ms":1e9,"spec":{"steps":10}}])");
  auto el = simulate_cluster(rows, 8, "ditserve", c);
  auto one = simulate_cluster(rows, 8, "xdit-sp1", c);
  CHECK(el.rows[0].at("finish_ms").as_double() < 0.25 * one.rows[0].at("finish_ms").as_double());
}

TEST("ring forms are offered only when enabled and price the ring term") {
  ClusterCost c(profile());
  Json o = Json::object();
  auto plain = candidate_forms(policy_traits("abl-step-elastic"), c, "long", 8, o);
  for (const auto& f : plain) CHECK(f.ring == 1);
  auto all = enumerate_forms({1, 2, 4, 8}, true, true, 8);
  bool u2r2 = false;
  for (const auto& f : all) u2r2 = u2r2 || form_name(f) == "u2r2";
  CHECK(u2r2);
  Json pr = profile();
  pr["classes"]["long"]["ring_mb_per_step"] = 8000;
  ClusterCost r(pr);
  CHECK(r.terms("long", parse_form("u2r2")).ring > 0);
}

TEST("near-linear scaling starts videos on their widest efficient form") {
  Json pr = profile();
  // measured NVSwitch-like forms: per-GPU work within 5% from cfg2 to cfg2sp4
  pr["classes"]["vid"]["forms"] = Json::parse(R"({"cfg2":{"step_ms":400},"cfg2sp2":{"step_ms":205},
                                                  "cfg2sp4":{"step_ms":105}})");
  ClusterCost c(pr);
  auto forms = candidate_forms(policy_traits("ditserve-wide"), c, "vid", 8, Json::object());
  CHECK(!forms.empty());
  for (const auto& f : forms) CHECK(f.degree() == 8);
  auto p = cluster_plan(state(8, {req("a", "video", "vid", 0, 1e9), req("b", "video", "vid", 0, 1e9)}),
                        "ditserve-wide", c);
  CHECK(find(p, "a")->at("degree").as_int() == 8);
  CHECK(find(p, "b") == nullptr);  // serialised behind a, not squeezed onto a narrow group
  auto q = cluster_plan(state(8, {req("a", "video", "vid", 0, 1e9), req("b", "video", "vid", 0, 1e9)}),
                        "ditserve", c);
  CHECK(find(q, "b") != nullptr || find(q, "a")->at("degree").as_int() == 8);
  // poor scaling (PCIe-like): the floor stays at the narrowest form
  Json slow = profile(2.0);
  ClusterCost s(slow);
  auto narrow = candidate_forms(policy_traits("ditserve-wide"), s, "vid", 8, Json::object());
  CHECK(narrow.front().degree() == 2);
}

TEST("CFG fission runs a fold-eligible video on the conditional half of its group") {
  ClusterCost c(profile());
  auto v = suspended("v", "[2,3]", "cfg2", 6, 0);
  v["cfg_fold_eligible"] = true;
  auto p = cluster_plan(state(8, {v}), "ditserve-approx", c);
  const Json* a = find(p, "v");
  CHECK(a != nullptr);
  CHECK(a->at("group").size() == 1 && a->at("group")[0].as_int() == 2);
  CHECK(a->at("form").as_string() == "sp1" && a->at("fold").as_bool());
  CHECK(a->at("reason").as_string() == "fission");
  auto q = cluster_plan(state(8, {v}), "ditserve", c);  // exact policy: no fission
  CHECK(!find(q, "v")->contains("fold"));
  v["cfg_fold_eligible"] = false;
  auto r = cluster_plan(state(8, {v}), "ditserve-approx", c);
  CHECK(!find(r, "v")->contains("fold"));
}

TEST("late short requests keep their EDF position with late_short_ms") {
  ClusterCost c(profile());
  auto late_img = req("img", "image", "img", 0, 10);   // already late, 400 ms of work
  auto vid = req("v", "video", "vid", 0, 20000);
  auto p = cluster_plan(state(1, {late_img, vid}, {}, 100), "abl-step-elastic", c);
  CHECK(find(p, "v") != nullptr && find(p, "img") == nullptr);  // demoted behind the feasible video
  Json o = Json::object();
  o["late_short_ms"] = 1000;
  auto q = cluster_plan(state(1, {late_img, vid}, {}, 100), "abl-step-elastic", c, o);
  CHECK(find(q, "img") != nullptr);                             // short: keeps its EDF slot
}

TEST("load-adaptive forms: efficient CFG pairs under load, the usual choice when few videos run") {
  Json pr = profile();
  pr["classes"]["vid"]["forms"] = Json::parse(R"({"cfg2":{"step_ms":400},"cfg2sp2":{"step_ms":210},
                                                  "cfg2sp4":{"step_ms":110}})");
  ClusterCost c(pr);
  std::vector<Json> many;
  for (int k = 0; k < 6; ++k) many.push_back(req("v" + std::to_string(k), "video", "vid", 0, 1e9));
  auto p = cluster_plan(state(8, many), "ditserve-b200", c);
  CHECK(p.at("assignments").size() == 4);
  for (const auto& a : p.at("assignments").as_array()) CHECK(a.at("form").as_string() == "cfg2");
  auto q = cluster_plan(state(8, {req("a", "video", "vid", 0, 1e9)}), "ditserve-b200", c);
  CHECK(find(q, "a")->at("degree").as_int() == 8);  // alone: widened as usual
  // under load, feasibility is judged on the efficient form: 10 steps x 400 ms misses 3 s
  many.push_back(req("tight", "video", "vid", 0, 3000));
  auto r = cluster_plan(state(8, many), "ditserve-b200", c);
  CHECK(find(r, "tight") == nullptr);               // demoted behind the feasible ones
}

TEST("a running lockstep pair is one preemption candidate") {
  ClusterCost c(profile());
  auto a = req("a", "video", "vid", 0, 1e9, 2);
  auto b = req("b", "video", "vid", 0, 1e9, 2);
  for (Json* r : {&a, &b}) {
    (*r)["status"] = "running";
    (*r)["group"] = Json::parse("[0]");
    (*r)["form"] = "sp1";
    (*r)["quantum_started_ms"] = 0.0;
  }
  auto i = req("i", "image", "img", 0, 800);
  auto p = cluster_plan(state(1, {a, b, i}, {0}), "ditserve", c);  // must not throw on the shared group
  CHECK(p.at("preempt").size() == 1);
}

int main() { return dstest::run_all(); }

TEST("multi-video guard: one video does not widen to its deadline at the cost of two feasible ones") {
  ClusterCost c(profile());  // cfg2 4100 ms, cfg2sp2 2222 ms, cfg2sp4 1215 ms to finish
  std::vector<Json> rs = {req("v0", "video", "vid", 0, 1500)};  // only cfg2sp4 (8 GPUs) meets it
  for (int k = 1; k <= 3; ++k) rs.push_back(req("v" + std::to_string(k), "video", "vid", 0, 5000));
  auto p = cluster_plan(state(8, rs), "ditserve", c);
  CHECK(p.at("assignments").size() == 4);
  CHECK(find(p, "v0")->at("degree").as_int() == 2);
  CHECK(find(p, "v0")->at("reason").as_string() == "multi-video-guard");
  auto lone = cluster_plan(state(8, {rs[0]}), "ditserve", c);
  CHECK(find(lone, "v0")->at("degree").as_int() == 8);  // nobody to protect: it widens
  Json off = Json::object();
  off["feasibility_guards"] = false;
  auto q = cluster_plan(state(8, rs), "ditserve", c, off);
  CHECK(find(q, "v0")->at("degree").as_int() == 8 && q.at("assignments").size() == 1);
}

TEST("threshold widening never costs a feasible video its GPUs") {
  ClusterCost c(profile());  // cfg2 -> cfg2sp2 keeps 94 % per-GPU efficiency (above 0.90)
  std::vector<Json> rs;
  for (int k = 0; k < 4; ++k) rs.push_back(req("v" + std::to_string(k), "video", "vid", 0, 5000 + k));
  auto p = cluster_plan(state(8, rs), "ditserve", c);
  CHECK(p.at("assignments").size() == 4);
  for (const auto& a : p.at("assignments").as_array()) CHECK(a.at("degree").as_int() == 2);
}

TEST("idle widening takes GPUs nobody else needs, below the efficiency threshold") {
  Json pr = profile();
  pr["classes"]["vid"]["forms"] = Json::parse(R"({"cfg2sp2":{"step_ms":300},"sp4":{"step_ms":320}})");  // 67 %
  ClusterCost c(pr);
  std::vector<Json> rs = {req("v0", "video", "vid", 0, 1e9), req("v1", "video", "vid", 0, 1e9 + 1)};
  auto p = cluster_plan(state(8, rs), "ditserve", c);
  CHECK(find(p, "v0")->at("degree").as_int() == 4 && find(p, "v0")->at("form").as_string() == "cfg2sp2");
  CHECK(find(p, "v0")->at("reason").as_string() == "idle-widened");
  CHECK(find(p, "v1")->at("degree").as_int() == 4);
  // three videos: the first may not take the pair the third needs
  rs.push_back(req("v2", "video", "vid", 0, 1e9 + 2));
  auto q = cluster_plan(state(8, rs), "ditserve", c);
  CHECK(q.at("assignments").size() == 3);
  CHECK(find(q, "v0")->at("degree").as_int() == 4 && find(q, "v1")->at("degree").as_int() == 2);
  Json off = Json::object();
  off["idle_widening"] = false;
  auto r = cluster_plan(state(8, {rs[0], rs[1]}), "ditserve", c, off);
  CHECK(find(r, "v0")->at("degree").as_int() == 2);
}

TEST("sunk-work deadband keeps an in-flight video's rank for a small overrun") {
  ClusterCost c(profile());
  Json in = suspended("in", "[0,1]", "cfg2", 6, 0);  // 4 steps + decode left: 1700 ms
  in["deadline_ms"] = 1500;                          // 200 ms over, under 15 % of 1700
  Json fresh = req("fresh", "video", "vid", 0, 1e5);
  auto p = cluster_plan(state(2, {in, fresh}), "ditserve", c);
  CHECK(find(p, "in") != nullptr && find(p, "fresh") == nullptr);
  // an unstarted video with a similar overrun is still demoted behind the feasible one
  Json un = req("un", "video", "vid", 0, 4000);      // needs 4100 ms
  auto q = cluster_plan(state(2, {un, fresh}), "ditserve", c);
  CHECK(find(q, "fresh") != nullptr && find(q, "un") == nullptr);
  // and a large overrun gets no deadband
  in["deadline_ms"] = 1000;
  auto r = cluster_plan(state(2, {in, fresh}), "ditserve", c);
  CHECK(find(r, "fresh") != nullptr && find(r, "in") == nullptr);
}

TEST("an image borrows the GPUs of the step-boundary video with the most laxity") {
  ClusterCost c(profile());
  Json urgent = suspended("urgent", "[0,1]", "cfg2", 2, 0);
  urgent["deadline_ms"] = 5000;   // 3300 ms left to run
  Json slack = suspended("slack", "[2,3]", "cfg2", 2, 0);
  slack["deadline_ms"] = 50000;
  Json img = req("img", "image", "img", 0, 2000);
  auto p = cluster_plan(state(4, {urgent, slack, img}), "ditserve", c);
  CHECK(find(p, "img")->at("group")[0].as_int() == 2);
  CHECK(find(p, "urgent")->at("group")[0].as_int() == 0 && !find(p, "urgent")->at("resize").as_bool());
  Json off = Json::object();
  off["feasibility_guards"] = false;
  auto q = cluster_plan(state(4, {urgent, slack, img}), "ditserve", c, off);
  CHECK(find(q, "img")->at("group")[0].as_int() == 0);
}

TEST("migration guard: a prepared video waits rather than reshard into lateness") {
  Json pr = profile();
  pr["resize_ms"] = 50;
  ClusterCost c(pr);
  Json v = suspended("v", "[0,1]", "cfg2", 9, 0);  // 400 + 100 ms left
  v["deadline_ms"] = 520;                          // on time in place, late after a 50 ms reshard
  auto p = cluster_plan(state(4, {v}, {0}), "ditserve", c);
  CHECK(find(p, "v") == nullptr);
  v["deadline_ms"] = 1e9;                          // plenty of slack: it moves
  auto q = cluster_plan(state(4, {v}, {0}), "ditserve", c);
  CHECK(find(q, "v") && find(q, "v")->at("group")[0].as_int() == 2 && find(q, "v")->at("resize").as_bool());
  Json off = Json::object();
  off["feasibility_guards"] = false;
  v["deadline_ms"] = 520;
  auto r = cluster_plan(state(4, {v}, {0}), "ditserve", c, off);
  CHECK(find(r, "v") != nullptr);
}

TEST("continuous batching belongs to the policy: baselines ignore the shared option") {
  ClusterCost c(profile());
  std::vector<Json> imgs = {req("i0", "image", "img", 0, 5000), req("i1", "image", "img", 0, 5000)};
  Json o = Json::object();
  o["continuous_batch"] = 4;
  auto d = cluster_plan(state(1, imgs), "ditserve", c, o);
  CHECK(d.at("assignments").size() == 1 && d.at("assignments")[0].at("quantum").as_string() == "continuous_batch");
  for (const char* base : {"abl-no-cb", "edf-bestfit", "tetriserve", "xdit-sp1", "edf-cfg2"}) {
    auto p = cluster_plan(state(2, imgs, {0}), base, c, o);
    CHECK(p.at("assignments").size() == 1);
    CHECK(p.at("assignments")[0].at("quantum").as_string() == "atomic");
  }
}

TEST("work-conserving continuous batching spreads waiting images over idle GPUs") {
  ClusterCost c(profile());
  std::vector<Json> two = {req("i0", "image", "img", 0, 5000), req("i1", "image", "img", 0, 5000)};
  auto p = cluster_plan(state(2, two), "ditserve", c);
  CHECK(p.at("assignments").size() == 2);
  for (const auto& a : p.at("assignments").as_array()) CHECK(a.at("batch").size() == 1);
  std::vector<Json> four = two;
  four.push_back(req("i2", "image", "img", 0, 5000));
  four.push_back(req("i3", "image", "img", 0, 5000));
  auto q = cluster_plan(state(2, four), "ditserve", c);
  CHECK(q.at("assignments").size() == 2);
  for (const auto& a : q.at("assignments").as_array()) CHECK(a.at("batch").size() == 2);
  // GPUs a waiting video needs are not counted as idle: four images share the two GPUs
  // that the video's CFG pair leaves
  std::vector<Json> mixed = four;
  mixed.push_back(req("v", "video", "vid", 0, 1e9));
  auto r = cluster_plan(state(4, mixed), "ditserve", c);
  CHECK(find(r, "i0")->at("batch").size() == 2);
  CHECK(find(r, "v") != nullptr && find(r, "v")->at("degree").as_int() == 2);
}

TEST("mixed-class continuous batches: order-free pricing and every member's deadline") {
  Json pr = profile();
  pr["classes"]["big"] = Json::parse(R"({"kind":"image","steps":28,"tokens":4096,"step_ms":40,"service_ms":1300,
                                         "decode_ms":180,"batch_step_ms":{"1":40,"2":74,"4":142,"8":280}})");
  ClusterCost c(pr);
  Json small = req("s", "image", "img", 0, 28 * 12 + 50 + 20);  // only alone keeps this deadline
  Json big = req("b", "image", "big", 0, 1e6);
  CHECK(std::abs(c.continuous_batch_step_ms({&small, &big}, true, "img") -
                 c.continuous_batch_step_ms({&big, &small}, true, "big")) < 1e-9);
  CHECK(c.batch_anchor({&small, &big}, "img") == "big");
  auto p = cluster_plan(state(1, {small, big}), "ditserve", c);
  CHECK(find(p, "s")->at("batch").size() == 1);  // the big member would make the small one late
  Json relaxed = small;
  relaxed["deadline_ms"] = 1e6;
  auto q = cluster_plan(state(1, {relaxed, big}), "ditserve", c);
  CHECK(q.at("assignments").size() == 1);  // sequence packing joins the two classes
  CHECK(q.at("assignments")[0].at("batch").size() == 2);
}

TEST("bubble-free batches hide member prepare and finish; without it they stall the round") {
  Json pr = profile();
  pr["classes"]["img"]["prepare_ms"] = 30;
  pr["classes"]["img"]["finish_ms"] = 30;
  ClusterCost c(pr);
  // one new member joining an almost finished batch: its prepare would stall every round
  Json a = req("a", "image", "img", 0, 28 * 16 + 50 + 20);   // fits a pair batch only when rounds are not stalled
  Json b = req("b", "image", "img", 0, 1e6);
  auto p = cluster_plan(state(1, {a, b}), "ditserve", c);
  CHECK(p.at("assignments").size() == 1 && p.at("assignments")[0].at("batch").size() == 2);
  CHECK(p.at("assignments")[0].at("bubble_free").as_bool());
  CHECK(p.at("assignments")[0].at("sequence_packing").as_bool());
  Json o = Json::object();
  o["bubble_free"] = false;
  auto q = cluster_plan(state(1, {a, b}), "ditserve", c, o);
  CHECK(q.at("assignments")[0].at("batch").size() == 1);
  CHECK(!q.at("assignments")[0].at("bubble_free").as_bool());
}

TEST("every policy resumes a mid-step request only on its own group and form") {
  ClusterCost c(profile());
  auto v = suspended("v", "[2,3]", "sp2", 3, 12);
  for (const char* pol : {"xdit-sp2", "tetriserve", "edf-bestfit", "sbp-esp", "ditserve-v1", "ditserve"}) {
    auto p = cluster_plan(state(8, {v}), pol, c);
    const Json* a = find(p, "v");
    CHECK(a != nullptr);
    CHECK(a->at("group")[0].as_int() == 2 && a->at("group")[1].as_int() == 3);
    CHECK(a->at("form").as_string() == "sp2");
    auto q = cluster_plan(state(8, {v}, {3}), pol, c);
    CHECK(find(q, "v") == nullptr);  // its GPU 3 is busy: wait, never move mid-step
  }
}

TEST("an xDiT partition on two GPUs keeps one GPU for videos and one for images") {
  ClusterCost c(profile());
  auto p = cluster_plan(state(2, {req("v", "video", "vid", 0, 1e9), req("w", "video", "vid", 0, 1e9 + 1)}),
                        "xdit-sp1", c);
  CHECK(p.at("assignments").size() == 1);
  CHECK(find(p, "v")->at("group")[0].as_int() == 0);
  auto q = cluster_plan(state(2, {req("i", "image", "img", 0, 5000), req("v", "video", "vid", 0, 1e9)}),
                        "xdit", c);
  CHECK(find(q, "i")->at("group")[0].as_int() == 1 && find(q, "v")->at("group")[0].as_int() == 0);
}

TEST("a video does not take GPUs another video holds inside a solver step") {
  ClusterCost c(profile());
  auto held = suspended("held", "[2,3]", "cfg2", 3, 12);  // mid-step on {2,3}, ranked second
  held["deadline_ms"] = 2e9;
  auto b = suspended("b", "[0,1]", "cfg2", 3, 0);         // at a step boundary; GPU 0 is busy
  for (const char* pol : {"ditserve", "edf-bestfit", "tetriserve"}) {
    auto p = cluster_plan(state(4, {b, held}, {0}), pol, c);
    CHECK(find(p, "held") != nullptr && find(p, "held")->at("group")[0].as_int() == 2);
    if (const Json* a = find(p, "b"))  // {2,3} is free but belongs to the mid-step video
      for (const auto& i : a->at("group").as_array()) CHECK(i.as_int() < 2);
  }
  // an image may still use it: the doorbell stopped the video for images
  auto q = cluster_plan(state(4, {held, req("i", "image", "img", 0, 5000)}, {0, 1, 3}), "ditserve", c);
  CHECK(find(q, "i") && find(q, "i")->at("group")[0].as_int() == 2);
}

TEST("deadline doorbells: a group's own timing, natural boundaries and already-rung capacity") {
  // {id, GPUs, stop_ms, remaining_ms, resume_ms, rung}
  const std::vector<RunningGroup> hetero = {{"fast-expensive", {0}, 10, 100, 1000, false},
                                           {"slow-cheap", {1}, 30, 200, 0, false}};
  auto sel = select_deadline_preemption(0, {{-1, 60, 40}}, hetero);
  CHECK(sel.selected == std::vector<std::string>{"fast-expensive"});  // only its stop saves the image
  CHECK(select_deadline_preemption(0, {{1, 60, 40}}, hetero).selected.empty());  // pinned to the slow one
  const std::vector<RunningGroup> boundary = {{"natural-boundary", {0}, 5, 5, 0, false},
                                              {"interrupt", {1}, 10, 100, 0, false}};
  CHECK(select_deadline_preemption(0, {{-1, 60, 40}}, boundary).selected.empty());  // a step ends in time
  const std::vector<RunningGroup> pending = {{"already-rung", {0, 1}, 5, 100, 0, true},
                                             {"extra", {2}, 5, 100, 0, false}};
  CHECK(select_deadline_preemption(0, {{-1, 50, 40}, {-1, 50, 40}}, pending).selected.empty());
}

TEST("an asynchronous decode keeps new videos off its GPU but lets images overlap") {
  ClusterCost c(profile());
  Json st = state(2, {req("a", "video", "vid", 0, 1e9), req("b", "video", "vid", 0, 1e9 + 1)});
  st["async_decoding"] = Json::parse("[true, false]");
  Json o = Json::object();
  o["degrees"] = Json::parse("[1]");
  auto p = cluster_plan(st, "abl-step-elastic", c, o);
  CHECK(p.at("assignments").size() == 1 && p.at("assignments")[0].at("group")[0].as_int() == 1);
  Json si = state(2, {req("i", "image", "img", 0, 5000)});
  si["async_decoding"] = Json::parse("[true, false]");
  auto q = cluster_plan(si, "static-sp1", c);
  CHECK(q.at("assignments").size() == 1 && q.at("assignments")[0].at("group")[0].as_int() == 0);
}

TEST("lazy block preemption: a new image waits for a mid-step video's boundary when it can") {
  ClusterCost c(profile());
  auto v = suspended("v", "[0,1]", "cfg2", 3, 15);  // 15 of 30 blocks left: 200 ms to its boundary
  Json relaxed = req("i", "image", "img", 0, 1000);   // 386 ms of work, 614 ms of slack
  auto p = cluster_plan(state(2, {v, relaxed}), "ditserve", c);
  CHECK(find(p, "v") != nullptr && find(p, "i") == nullptr);
  Json tight = req("i", "image", "img", 0, 500);      // 114 ms of slack: it takes the GPU now
  auto q = cluster_plan(state(2, {v, tight}), "ditserve", c);
  CHECK(find(q, "i") != nullptr && find(q, "v") == nullptr);
  Json o = Json::object();
  o["lazy_preemption"] = false;
  auto r = cluster_plan(state(2, {v, relaxed}), "ditserve", c, o);
  CHECK(find(r, "i") != nullptr);
}

TEST("lateness is judged on the widest group free when the plan starts (elastic policies)") {
  ClusterCost c(profile());
  Json v = req("v", "video", "vid", 0, 3000);  // cfg2sp2 (2222 ms) or wider meets it; cfg2 (4100) does not
  auto feasible_in = [&](const Json& o) {
    PlanTrace tr;
    cluster_plan(state(8, {v}, {0, 1, 2, 3, 4, 5}), "ditserve", c, o, &tr);
    return tr.rows[0].at("feasible").as_bool();
  };
  CHECK(!feasible_in(Json::object()));  // only a pair is free
  Json widest = Json::object();
  widest["feasibility_degree"] = "widest";
  CHECK(feasible_in(widest));
  PlanTrace tr;
  cluster_plan(state(8, {v}), "ditserve", c, Json::object(), &tr);
  CHECK(tr.rows[0].at("feasible").as_bool());  // an idle node
}

TEST("quantum_ms sizes block quanta by GPU time and never crosses the step boundary") {
  ClusterCost c(profile());  // cfg2: 400 ms per 30-block step
  Json o = Json::object();
  o["quantum_ms"] = 100;
  auto p = cluster_plan(state(2, {req("v", "video", "vid", 0, 1e9)}), "ditserve", c, o);
  CHECK(find(p, "v")->at("quantum").as_int() == 7);
  auto m = suspended("m", "[0,1]", "cfg2", 3, 28);
  auto q = cluster_plan(state(2, {m}), "ditserve", c, o);
  CHECK(find(q, "m")->at("quantum").as_int() == 2);
  o["quantum_ms"] = 1e100;
  auto r = cluster_plan(state(2, {req("v", "video", "vid", 0, 1e9)}), "ditserve", c, o);
  CHECK(find(r, "v")->at("quantum").as_int() == 30);
}

TEST("late images share continuous batches under ditserve-b200; on-time images run alone") {
  ClusterCost c(profile());
  // img: 28 steps x 12 ms + 50 ms decode = 386 ms alone
  std::vector<Json> late = {req("l0", "image", "img", 0, 100), req("l1", "image", "img", 0, 100),
                            req("l2", "image", "img", 0, 100)};
  auto p = cluster_plan(state(1, late), "ditserve-b200", c);
  CHECK(p.at("assignments").size() == 1 && p.at("assignments")[0].at("quantum").as_string() == "continuous_batch");
  CHECK(p.at("assignments")[0].at("batch").size() == 3);
  std::vector<Json> fine = {req("f0", "image", "img", 0, 5000), req("f1", "image", "img", 0, 5000)};
  auto q = cluster_plan(state(1, fine), "ditserve-b200", c);
  CHECK(q.at("assignments").size() == 1 && q.at("assignments")[0].at("quantum").as_string() == "atomic");
  Json off = Json::object();
  off["late_image_batching"] = false;
  auto r = cluster_plan(state(1, late), "ditserve-b200", c, off);
  CHECK(r.at("assignments")[0].at("quantum").as_string() == "atomic");
}

TEST("fission: an urgent image takes the companion GPU while the folded video keeps its primary") {
  ClusterCost c(profile());
  Json v = suspended("v", "[0,1]", "cfg2", 6, 0);
  v["cfg_fold_eligible"] = true;
  Json img = req("i", "image", "img", 0, 500);
  auto p = cluster_plan(state(2, {v, img}), "ditserve-approx", c);
  CHECK(find(p, "i") && find(p, "i")->at("group")[0].as_int() == 1);
  CHECK(find(p, "v") && find(p, "v")->at("group")[0].as_int() == 0 && find(p, "v")->at("degree").as_int() == 1);
  CHECK(find(p, "v")->at("reason").as_string() == "fission");
}

TEST("feasibility counts the dispatch overhead of the quanta still to run") {
  Json pr = profile();
  pr["quantum_overhead_ms"] = 10;
  ClusterCost c(pr);  // cfg2: 10 steps x 400 ms + 100 ms decode = 4100 ms, 11 quanta
  Json v = req("v", "video", "vid", 0, 4150);
  auto feasible = [&](const Json& o) {
    PlanTrace tr;
    cluster_plan(state(2, {v}), "ditserve", c, o, &tr);
    return tr.rows[0].at("feasible").as_bool();
  };
  CHECK(!feasible(Json::object()));          // 4100 + 11 x 10 > 4150
  v["deadline_ms"] = 4250;
  CHECK(feasible(Json::object()));           // 4210 <= 4250
  Json blocks = Json::object();
  blocks["quantum_blocks"] = 4;              // 8 block quanta per step: 81 quanta, 4910 ms
  CHECK(!feasible(blocks));
}
