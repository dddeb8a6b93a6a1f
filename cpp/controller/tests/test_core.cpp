// JSON, RNG, forms, policies, workload/metrics/gates/matrix, cost model, budget ledger.
#include <unistd.h>

#include <cstdio>
#include <set>

#include "check.hpp"
#include "ds/budget.hpp"
#include "ds/cost.hpp"
#include "ds/json.hpp"
#include "ds/policy.hpp"
#include "ds/rng.hpp"
#include "ds/study.hpp"
#include "ds/workload.hpp"

using namespace ds;

TEST("json round trip and strictness") {
  Json j = Json::parse(R"({"b":[1,2.5,"x\n",true,null],"a":{"k":-3e2}})");
  CHECK(j.at("b")[0].is_integer());
  CHECK(j.at("b")[1].as_double() == 2.5);
  CHECK(j.at("a").at("k").as_double() == -300.0);
  CHECK(Json::parse(j.dump()) == j);
  CHECK(j.dump() == R"({"a":{"k":-300.0},"b":[1,2.5,"x\n",true,null]})");
  CHECK_THROWS(Json::parse("NaN"));
  CHECK_THROWS(Json::parse(R"({"a":1,"a":2})"));
  CHECK_THROWS(Json::parse("[1,]"));
  CHECK_THROWS(Json::parse("{} x"));
  CHECK_THROWS(Json::parse("\"\x01\""));
  CHECK(Json::parse(R"("é😀")").as_string() == "\xc3\xa9\xf0\x9f\x98\x80");
  CHECK_THROWS(Json(1.0 / 0.0));
}

TEST("rng determinism and bit-exact snapshot") {
  Random a(42), b(42);
  for (int i = 0; i < 100; ++i) CHECK(a.next_u64() == b.next_u64());
  a.normal();  // leaves a cached spare
  Json snap = a.snapshot();
  std::vector<double> want;
  for (int i = 0; i < 10; ++i) want.push_back(a.normal() + a.exponential(2.0) + a.gamma(0.5, 1.0));
  Random c(0);
  c.restore(snap);
  for (int i = 0; i < 10; ++i) CHECK(c.normal() + c.exponential(2.0) + c.gamma(0.5, 1.0) == want[i]);
  Random d(7);
  std::vector<int> counts(6, 0);
  for (int i = 0; i < 60000; ++i) ++counts[d.below(6)];
  for (int k : counts) CHECK(k > 9000 && k < 11000);
  CHECK_THROWS(d.below(0));
  double m = 0;
  for (int i = 0; i < 20000; ++i) m += d.gamma(2.0, 3.0);
  CHECK_NEAR(m / 20000, 6.0, 0.2);
}

TEST("form names") {
  for (const char* n : {"sp1", "sp2", "sp4", "sp8", "cfg2", "cfg2sp2", "cfg2sp4", "u2r2", "u4r2", "cfg2u2r2", "sp3", "sp6"})
    CHECK(form_name(parse_form(n)) == n);
  CHECK(parse_form("cfg2sp4").degree() == 8);
  CHECK(parse_form("u2r2").sp == 4 && parse_form("u2r2").ring == 2);
  CHECK_THROWS(parse_form("u1r2"));
  CHECK_THROWS(parse_form("spx"));
  CHECK_THROWS(parse_form("cfg3"));
}

TEST("policy registry") {
  const auto cat = policy_catalog();
  std::set<std::string> ids;
  for (const auto& p : cat.as_array()) ids.insert(p.at("id").as_string());
  for (const char* id : {"ditserve", "ditserve-approx", "tetriserve", "sbp-esp", "edf-bestfit", "edf-cfg2", "cfg2-first",
                         "partition", "abl-no-block", "stair-base", "ditserve-v1", "diag-2d-usp", "xdit-sp1"})
    CHECK(ids.count(id));
  CHECK(policy_traits("ditserve").blocks && policy_traits("ditserve").min_video_degree == 2);
  CHECK(!policy_traits("abl-no-block").blocks);
  CHECK(policy_traits("edf-bestfit").best_fit && !policy_traits("edf-bestfit").demote_late);
  CHECK(policy_traits("static-cfg2sp4").fixed_degree == 8);
  CHECK(policy_traits("xdit").order == "fcfs");
  CHECK(canonical_policy("step_elastic") == "abl-step-elastic");
  CHECK(canonical_policy("static_sp2") == "static-sp2");
  CHECK_THROWS(policy_traits("vanilla_xdit"));
  CHECK_THROWS(policy_traits("nope"));
}

TEST("workload generator is seeded and class mixtures do not move arrivals") {
  Json g = Json::parse(R"({"generator":{"count":50,"seed":3,"pattern":"poisson","rate_rpm":2,
      "classes":[{"weight":2,"kind":"video","class":"wan21_480p","service_ms":1000,"slo_scale_range":[1.5,3]},
                 {"weight":1,"kind":"image","class":"sd35_512","service_ms":100,"slo_scale":2}]}})");
  Json a = study_workload(g), b = study_workload(g);
  CHECK(a == b);
  Json g2 = g;
  g2["generator"]["classes"][1]["weight"] = 5;
  Json c = study_workload(g2);
  for (size_t i = 0; i < a.size(); ++i) CHECK(a[i].at("arrival_ms") == c[i].at("arrival_ms"));
  double last = -1;
  int videos = 0;
  for (const auto& r : a.as_array()) {
    CHECK(r.at("arrival_ms").as_double() >= last);
    last = r.at("arrival_ms").as_double();
    const double slo = r.at("slo_ms").as_double() / r.at("service_ms").as_double();
    if (r.at("kind").as_string() == "video") {
      ++videos;
      CHECK(slo >= 1.5 && slo <= 3.0);
    }
  }
  CHECK(videos > 20 && videos < 45);
  CHECK_NEAR(last / 49.0, 30000.0, 12000.0);  // mean gap of 2 rpm
  for (const char* p : {"offline_all", "steady", "bursty", "gamma"}) {
    Json h = g;
    h["generator"]["pattern"] = p;
    CHECK(study_workload(h).size() == 50);
  }
  Json bad = g;
  bad["generator"]["pattern"] = "zipf";
  CHECK_THROWS(study_workload(bad));
}

TEST("summary counts failed and unfinished requests in the denominator") {
  Json rows = Json::parse(R"([
    {"request_id":"a","kind":"video","arrival_ms":0,"deadline_ms":100,"status":"done","finish_ms":90},
    {"request_id":"b","kind":"video","arrival_ms":0,"deadline_ms":100,"status":"done","finish_ms":150},
    {"request_id":"c","kind":"image","arrival_ms":10,"deadline_ms":50,"status":"failed"},
    {"request_id":"d","kind":"image","arrival_ms":10,"deadline_ms":50,"status":"done","finish_ms":40}])");
  Json s = request_summary(rows);
  CHECK(s.at("requests").as_int() == 4);
  CHECK(s.at("on_time").as_int() == 2);
  CHECK_NEAR(s.at("slo_attainment").as_double(), 0.5, 1e-12);
  CHECK_NEAR(s.at("goodput_rps").as_double(), 2 / 0.15, 1e-9);
  CHECK_NEAR(s.at("kinds").at("image").at("slo_attainment").as_double(), 0.5, 1e-12);
  CHECK_NEAR(s.at("latency_p50_ms").as_double(), 90.0, 1e-9);
}

TEST("gates and matrix") {
  Json ev = Json::parse(R"({"summary":{"sar":0.93,"name":"x"}})");
  Json rules = Json::parse(R"([{"pointer":"/summary/sar","op":">=","value":0.9},
                               {"pointer":"/summary/name","op":"==","value":"x"}])");
  CHECK(evaluate_gates(ev, rules).at("pass").as_bool());
  rules[0]["value"] = 0.95;
  CHECK(!evaluate_gates(ev, rules).at("pass").as_bool());
  Json missing = Json::parse(R"([{"pointer":"/nope","op":">","value":1}])");
  CHECK(!evaluate_gates(ev, missing).at("pass").as_bool());
  Json ph = Json::parse(R"({"id":"p","policy":"edf","matrix":{"axes":[{"pointer":"/policy","values":["fcfs","edf"]},
                          {"pointer":"/options/seed","values":[1,2,3]}]}})");
  Json cells = expand_matrix(ph);
  CHECK(cells.size() == 6);
  CHECK(cells[5].at("policy").as_string() == "edf" && cells[5].at("options").at("seed").as_int() == 3);
  Json ph2 = Json::parse(R"({"id":"p","matrix":{"/policy":["fcfs","edf","srtf"]}})");
  CHECK(expand_matrix(ph2).size() == 3);
}

TEST("cost model formula and measured overrides") {
  Json p = Json::parse(R"({"classes":{"v":{"kind":"video","steps":10,"blocks_per_step":30,
      "step_compute_ms":800,"comm_mb_per_step":7000,"collectives_per_step":100,"cfg_exchange_mb":70,
      "forms":{"cfg2sp4":{"step_ms":111}}},
      "i":{"kind":"image","steps":20,"service_ms":400,"decode_ms":40,"batch_step_ms":{"1":18,"4":40}}},
      "links":{"default_gbps":700,"default_latency_ms":0.01}})");
  ClusterCost c(p);
  CHECK_NEAR(c.step_ms("v", parse_form("sp1")), 800.0, 1e-9);
  // sp2: 400 + 7000*(1/4)/700 + 100*0.01
  CHECK_NEAR(c.step_ms("v", parse_form("sp2")), 400.0 + 2.5 + 1.0, 1e-9);
  // cfg2: 400 + 70/700 + 0.01
  CHECK_NEAR(c.step_ms("v", parse_form("cfg2")), 400.0 + 0.1 + 0.01, 1e-9);
  CHECK_NEAR(c.step_ms("v", parse_form("cfg2sp4")), 111.0, 1e-9);
  Json r = Json::parse(R"({"class":"v","steps_done":4,"blocks_done":15})");
  CHECK_NEAR(c.remaining_ms(r, parse_form("sp1")), 6 * 800.0 - 15 * 800.0 / 30, 1e-6);
  CHECK_NEAR(c.continuous_step_ms("i", 2.5), 18 + (40 - 18) * 0.5, 1e-9);
  CHECK_NEAR(c.image_step_ms("i"), (400 - 40) / 20.0, 1e-9);
  CHECK_THROWS(ClusterCost(Json::parse(R"({"classes":{"x":{"kind":"other"}}})")));
}

TEST("budget ledger: sessions, deadlines, poisoning and repair") {
  char tmpl[] = "/tmp/dsbudgetXXXXXX";
  const std::string dir = mkdtemp(tmpl);
  const std::string path = dir + "/ledger.json";
  double now = 1000.0;
  auto clock = [&]() { return now; };
  Json limits = Json::parse(R"({"phases":{"a":{"gpu_seconds":100},"b":{"gpu_seconds":50}},"carry":"forward",
                               "repair_reserve_gpu_seconds":40})");
  {
    Budget b(path, limits, clock);
    CHECK_THROWS(Budget(path, limits, clock));  // flock held
    b.begin("run1/a", 2, "a", 0);
    CHECK_NEAR(b.deadline(), 1000.0 + 50.0, 1e-9);
    now += 10;
    b.check();
    auto s = b.finish("ok", true);
    CHECK_NEAR(s.at("gpu_seconds").as_double(), 20.0, 1e-9);
    CHECK_NEAR(b.allowance("a"), 80.0, 1e-9);
    CHECK_NEAR(b.allowance("b"), 130.0, 1e-9);  // carry forward of a's unused 80
    b.begin("run1/b", 1, "b", 5);
    now += 6;
    CHECK_THROWS(b.check());
    b.finish("failed", false);
    CHECK(b.poisoned());
    CHECK_THROWS(b.begin("run2/a", 1, "a", 0));
    b.begin("repair", 1, "a", 0, true);
    now += 1;
    b.finish("ok", true);
    CHECK(!b.poisoned());
  }
  {
    Budget again(path, limits, clock);  // re-validates history
    CHECK(again.ledger().at("sessions").size() == 3);
  }
  std::remove(path.c_str());
  std::remove((path + ".lock").c_str());
  rmdir(dir.c_str());
}

TEST("select_action orders") {
  Json rows = Json::parse(R"([{"request_id":"a","arrival_ms":0,"deadline_ms":900,"remaining_ms":50},
                              {"request_id":"b","arrival_ms":5,"deadline_ms":300,"remaining_ms":500},
                              {"request_id":"c","arrival_ms":1,"deadline_ms":600,"remaining_ms":10}])");
  CHECK(select_action(rows, 10, "fcfs").at("request_id").as_string() == "a");
  CHECK(select_action(rows, 10, "edf").at("request_id").as_string() == "b");
  CHECK(select_action(rows, 10, "srtf").at("request_id").as_string() == "c");
  CHECK_THROWS(select_action(rows, 10, "lifo"));
}

int main() { return dstest::run_all(); }
