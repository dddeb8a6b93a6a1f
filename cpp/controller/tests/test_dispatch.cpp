// Online single-worker selection: benchmark orders, session policies, EDF arms, guarded arms.
#include "check.hpp"
#include "ds/dispatch.hpp"

using namespace ds;

namespace {

// a denoise row with a per-step cost table
Json row(const std::string& id, double arrival, double deadline, double remaining, double service = 100,
         double ready_since = -1, const char* kind = "video", double per_step = 10, bool started = false) {
  Json r = Json::object();
  r["request_id"] = id;
  r["kind"] = kind;
  r["arrival_ms"] = arrival;
  r["deadline_ms"] = deadline;
  r["remaining_ms"] = remaining;
  r["service_ms"] = service;
  r["ready_since_ms"] = ready_since < 0 ? arrival : ready_since;
  r["action"] = std::string(kind) == "image" ? "image" : "denoise";
  r["started"] = started;
  Json t = Json::object();
  for (int q : {1, 2, 4, 8}) t[std::to_string(q)] = per_step * q;
  t["step"] = per_step;
  r["action_ms_by_quantum"] = t;
  r["ready"] = true;
  r["release_ms"] = arrival;
  r["stage_deadline_ms"] = deadline;
  r["remaining_total_ms"] = remaining;
  return r;
}

Json arr(std::initializer_list<Json> xs) {
  Json a = Json::array();
  for (const auto& x : xs) a.push_back(x);
  return a;
}

std::string pick(const Json& d) { return d.at("request_id").is_null() ? "" : d.at("request_id").as_string(); }

}  // namespace

TEST("benchmark orders keep the active request unless another strictly precedes it") {
  Json rows = arr({row("a", 0, 900, 50), row("b", 5, 300, 500), row("c", 1, 600, 10)});
  CHECK(pick(select_online(rows, 10, "fcfs")) == "a");
  CHECK(pick(select_online(rows, 10, "edf")) == "b");
  CHECK(pick(select_online(rows, 10, "srtf")) == "c");
  CHECK(pick(select_online(rows, 10, "fcfs", "c")) == "c");   // fcfs never switches away
  CHECK(pick(select_online(rows, 10, "edf", "c")) == "b");    // b's deadline strictly earlier
  Json tie = arr({row("a", 0, 300, 50), row("b", 5, 300, 500)});
  CHECK(pick(select_online(tie, 10, "edf", "b")) == "b");      // equal deadline: stay
}

TEST("session policies: serial stickiness, stage deadline, least slack") {
  Json a = row("a", 0, 1000, 100), b = row("b", 0, 800, 700);
  a["stage_deadline_ms"] = 200;
  Json rows = arr({a, b});
  CHECK(pick(select_online(rows, 10, "session_serial", "a")) == "a");
  CHECK(pick(select_online(rows, 10, "session_serial")) == "b");  // no active: earliest deadline
  CHECK(pick(select_online(rows, 10, "stage_edf")) == "a");
  CHECK(pick(select_online(rows, 10, "session_slack")) == "b");   // slack 90 vs 890
}

TEST("EDF arms use their fixed quantum") {
  Json rows = arr({row("a", 0, 900, 50), row("b", 0, 300, 50)});
  auto d = select_online(rows, 10, "edf_b4");
  CHECK(pick(d) == "b" && d.at("quantum").as_int() == 4 && d.at("reason").as_string() == "edf");
  CHECK(select_online(rows, 10, "edf_b2").at("quantum").as_int() == 2);
  CHECK(select_online(rows, 10, "edf_b1_async").at("quantum").as_int() == 1);
  CHECK(select_online(rows, 10, "edf_step").at("quantum").as_string() == "step");
}

TEST("waiting guard serves a long-waiting request unless it endangers a deadline") {
  // w has waited 300 ms >= 2.5 x 100 ms of service; e has slack 1000
  Json rows = arr({row("w", 0, 5000, 100, 100, 0), row("e", 0, 1300, 100, 100, 290)});
  auto d = select_online(rows, 300, "feasible_b4");
  CHECK(pick(d) == "w" && d.at("reason").as_string() == "waiting_guard");
  // now e's slack (40 ms) is below w's quantum cost (40 = 4 x 10 ms)? make it smaller: 30 ms
  Json tight = arr({row("w", 0, 5000, 100, 100, 0), row("e", 0, 430, 100, 100, 290)});
  auto t = select_online(tight, 300, "feasible_b4");
  CHECK(pick(t) == "e" && t.at("reason").as_string() == "deadline_conflict_edf_min_quantum");
  CHECK(t.at("quantum").as_int() == 1 && t.at("predicted_deadline_conflict").as_bool());
}

TEST("feasible EDF skips a request that can no longer make its deadline") {
  Json rows = arr({row("late", 0, 100, 500, 600), row("ok", 0, 2000, 100, 600)});
  auto d = select_online(rows, 10, "feasible_b4");
  CHECK(pick(d) == "ok" && d.at("reason").as_string() == "feasible_edf");
  Json all_late = arr({row("x", 0, 100, 500, 600), row("y", 0, 50, 500, 600)});
  CHECK(select_online(all_late, 10, "feasible_b4").at("reason").as_string() == "edf_all_predicted_late");
}

TEST("resume guard lets a started video with thin slack go first") {
  // candidate c (earliest deadline, slack 500) would spend 40 ms; started video v has slack 30
  Json rows = arr({row("c", 0, 600, 90, 600, 5), row("v", 0, 700, 660, 600, 5, "video", 5, true)});
  auto d = select_online(rows, 10, "guarded_b4");
  CHECK(pick(d) == "v" && d.at("reason").as_string() == "video_resume_guard");
  auto f = select_online(rows, 10, "feasible_b4");                 // feasible arm has no resume guard
  CHECK(pick(f) != "v" || f.at("reason").as_string() != "video_resume_guard");
}

TEST("adaptive quantum: the largest of 1/4/8 that fits the others' slack and half the image deadline") {
  Json costs = Json::parse(R"({"image_deadline_ms": 1000})");
  Json rows = arr({row("a", 0, 500, 100, 600), row("b", 0, 5000, 100, 600)});  // b slack 4890
  auto d = select_online(rows, 10, "guarded_adaptive", "", Json(1), costs);
  CHECK(pick(d) == "a" && d.at("quantum").as_int() == 8);         // 80 ms fits min(500, 4890)
  Json tight = arr({row("a", 0, 500, 100, 600), row("b", 0, 170, 100, 600)});  // b slack 60
  auto t = select_online(tight, 10, "guarded_adaptive", "", Json(1), costs);
  CHECK(pick(t) == "b");                                            // b is the feasible earliest deadline
  Json img = arr({row("i", 0, 500, 100, 600, -1, "image"), row("b", 0, 5000, 100, 600)});
  CHECK(select_online(img, 10, "guarded_adaptive", "", Json(1), costs).at("quantum").as_int() == 1);  // images: 1
}

TEST("no ready request and invalid input") {
  Json future = arr({row("a", 100, 900, 50)});
  CHECK(select_online(future, 10, "edf").at("request_id").is_null());
  CHECK_THROWS(select_online(arr({row("a", 0, 9, 1), row("a", 0, 9, 1)}), 10, "edf"));
  CHECK_THROWS(select_online(arr({row("a", 0, 9, 1)}), 10, "lifo"));
  Json bad = row("a", 0, 900, 50);
  bad["action"] = "dance";
  CHECK_THROWS(select_online(arr({bad}), 10, "guarded_b4"));
}

int main() { return dstest::run_all(); }
