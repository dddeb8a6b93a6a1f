#include "ds/dispatch.hpp"

#include <algorithm>
#include <cmath>
#include <set>
#include <stdexcept>
#include <tuple>
#include <vector>

namespace ds {
namespace {

const std::set<std::string>& benchmark_policies() {
  static const std::set<std::string> s = {"fcfs", "edf", "srtf"};
  return s;
}
const std::set<std::string>& session_policies() {
  static const std::set<std::string> s = {"session_serial", "stage_edf", "session_slack"};
  return s;
}
const std::set<std::string>& arm_policies() {
  static const std::set<std::string> s = {"edf_b1", "edf_b1_async", "edf_b2", "edf_b4", "edf_step",
                                          "guarded_b4", "guarded_adaptive", "feasible_b4"};
  return s;
}

double field(const Json& r, const char* key) {
  const Json& v = r.at(key);
  if (!v.is_number()) throw std::invalid_argument(std::string(key) + " must be numeric");
  const double x = v.as_double();
  if (!std::isfinite(x)) throw std::invalid_argument(std::string(key) + " must be finite");
  return x;
}

struct View {
  const Json* row;
  std::string id;
  double arrival, deadline, remaining;
};

double slack_of(const View& v, double now) { return v.deadline - now - v.remaining; }

std::string quantum_key(const Json& q) { return q.is_string() ? q.as_string() : std::to_string(q.as_int()); }

double cost_of(const View& v, const Json& q) {
  const Json& table = v.row->at("action_ms_by_quantum");
  const std::string k = quantum_key(q);
  if (!table.contains(k)) throw std::invalid_argument("no action cost for quantum " + k + " of " + v.id);
  return field(table, k.c_str());
}

auto edf_key(const View& v) { return std::make_tuple(v.deadline, v.arrival, v.id); }

// another deadline that can still be met would be missed if `cost` ms go to `chosen`
bool endangers(const std::vector<View>& rows, const View& chosen, double cost, double now) {
  for (const auto& r : rows) {
    if (r.id == chosen.id) continue;
    const double s = slack_of(r, now);
    if (s >= 0 && s < cost) return true;
  }
  return false;
}

// quantum for `v`: fixed, or (adaptive) the largest of {1, 4, 8} whose cost fits the others'
// smallest slack and half the image deadline; the bool says "even 1 does not fit"
std::pair<Json, bool> pick_quantum(const View& v, const std::vector<View>& rows, double now, const Json& q,
                                   const Json& costs) {
  if (!(q.is_string() && q.as_string() == "adaptive")) {
    cost_of(v, q);  // validates that the cost exists
    return {q, false};
  }
  double limit = 0.5 * field(costs, "image_deadline_ms");
  for (const auto& r : rows)
    if (r.id != v.id && slack_of(r, now) >= 0) limit = std::min(limit, slack_of(r, now));
  int best = 0;
  for (int size : {1, 4, 8}) {
    if (size > 1 && v.row->str("action", "") != "denoise") break;
    if (cost_of(v, Json(size)) <= limit) best = size;
  }
  return {Json(best ? best : 1), best == 0};
}

Json decide(const View& v, const Json& q, const std::string& reason, bool conflict, double now) {
  Json d = Json::object();
  d["request_id"] = v.id;
  d["quantum"] = q;
  d["reason"] = reason;
  d["predicted_deadline_conflict"] = conflict;
  d["slack_ms"] = slack_of(v, now);
  return d;
}

}  // namespace

bool is_online_policy(const std::string& p) {
  return benchmark_policies().count(p) || session_policies().count(p) || arm_policies().count(p);
}

Json select_online(const Json& input, double now, const std::string& policy, const std::string& active,
                   const Json& default_quantum, const Json& costs) {
  if (!std::isfinite(now)) throw std::invalid_argument("now_ms must be finite");
  if (!input.is_array()) throw std::invalid_argument("rows must be an array");
  if (!is_online_policy(policy)) throw std::invalid_argument("unknown online policy: " + policy);
  const bool session = session_policies().count(policy) > 0;
  const bool benchmark = benchmark_policies().count(policy) > 0;
  std::vector<View> rows;
  std::set<std::string> seen;
  for (const auto& r : input.as_array()) {
    const std::string status = r.str("status", "pending");
    if (status != "pending" && !(session && status == "running")) continue;
    if (session ? !r.flag("ready", false) : !(r.flag("arrived", true) && r.flag("gpu_ready", true))) continue;
    if (field(r, session ? "release_ms" : "arrival_ms") > now) continue;
    View v;
    v.row = &r;
    v.id = r.at("request_id").as_string();
    if (v.id.empty() || !seen.insert(v.id).second) throw std::invalid_argument("request ids must be unique and non-empty");
    v.deadline = field(r, "deadline_ms");
    if (session) {
      v.arrival = field(r, "release_ms");
      field(r, "stage_deadline_ms");
      v.remaining = field(r, "remaining_total_ms");
      if (v.deadline < v.arrival) throw std::invalid_argument("deadline precedes release");
    } else {
      v.arrival = field(r, "arrival_ms");
      v.remaining = field(r, "remaining_ms");
      if (!benchmark) {
        const double since = field(r, "ready_since_ms");
        if (since < v.arrival || since > now) throw std::invalid_argument("ready_since_ms outside [arrival, now]");
        if (field(r, "service_ms") <= 0) throw std::invalid_argument("service_ms must be positive");
        const std::string kind = r.str("kind", "");
        if (kind != "video" && kind != "image") throw std::invalid_argument("kind must be video or image");
        const std::string action = r.str("action", "");
        if (action != "prepare" && action != "denoise" && action != "decode" && action != "image")
          throw std::invalid_argument("unknown action " + action);
      }
    }
    rows.push_back(v);
  }
  if (rows.empty()) {
    Json d = Json::object();
    d["request_id"] = Json();
    d["quantum"] = Json();
    d["reason"] = "no_ready_request";
    d["predicted_deadline_conflict"] = false;
    d["slack_ms"] = Json();
    return d;
  }
  const View* current = nullptr;
  for (const auto& v : rows)
    if (v.id == active) current = &v;

  if (session) {
    auto key = [&](const View& v) {
      double primary = v.deadline;
      if (policy == "stage_edf") primary = field(*v.row, "stage_deadline_ms");
      if (policy == "session_slack") primary = slack_of(v, now);
      return std::make_tuple(primary, v.deadline, v.arrival, v.id);
    };
    const View* pick = &rows.front();
    for (const auto& v : rows)
      if (key(v) < key(*pick)) pick = &v;
    if (policy == "session_serial" && current) pick = current;
    return decide(*pick, default_quantum, policy, false, now);
  }

  if (benchmark) {
    auto prio = [&](const View& v) {
      return policy == "fcfs" ? v.arrival : policy == "edf" ? v.deadline : v.remaining;
    };
    auto key = [&](const View& v) { return std::make_tuple(prio(v), v.arrival, v.id); };
    const View* best = &rows.front();
    for (const auto& v : rows)
      if (key(v) < key(*best)) best = &v;
    if (current && (policy == "fcfs" || prio(*current) <= prio(*best))) best = current;
    return decide(*best, default_quantum, policy, false, now);
  }

  Json quantum = Json(4);
  if (policy == "edf_step") quantum = Json("step");
  else if (policy == "guarded_adaptive") quantum = Json("adaptive");
  else if (policy == "edf_b2") quantum = Json(2);
  else if (policy == "edf_b1" || policy == "edf_b1_async") quantum = Json(1);
  const View* earliest = &rows.front();
  for (const auto& v : rows)
    if (edf_key(v) < edf_key(*earliest)) earliest = &v;
  if (policy.rfind("edf", 0) == 0) {
    cost_of(*earliest, quantum);
    return decide(*earliest, quantum, "edf", false, now);
  }
  auto fallback = [&]() {
    cost_of(*earliest, Json(1));
    return decide(*earliest, Json(1), "deadline_conflict_edf_min_quantum", true, now);
  };
  // (a) waiting guard
  const View* waiting = nullptr;
  auto wait_key = [&](const View& v) {
    return std::make_tuple(field(*v.row, "ready_since_ms") + 2.5 * field(*v.row, "service_ms"), edf_key(v));
  };
  for (const auto& v : rows)
    if (now - field(*v.row, "ready_since_ms") >= 2.5 * field(*v.row, "service_ms") &&
        (!waiting || wait_key(v) < wait_key(*waiting)))
      waiting = &v;
  if (waiting) {
    const auto q = pick_quantum(*waiting, rows, now, quantum, costs);
    if (!q.second && !endangers(rows, *waiting, cost_of(*waiting, q.first), now))
      return decide(*waiting, q.first, "waiting_guard", false, now);
    return fallback();
  }
  // feasible EDF
  const View* candidate = nullptr;
  for (const auto& v : rows)
    if (slack_of(v, now) >= 0 && (!candidate || edf_key(v) < edf_key(*candidate))) candidate = &v;
  const std::string reason = candidate ? "feasible_edf" : "edf_all_predicted_late";
  if (!candidate) candidate = earliest;
  const auto q = pick_quantum(*candidate, rows, now, quantum, costs);
  const double cost = cost_of(*candidate, q.first);
  // (b) resume guard: a started video that would lose its deadline behind the candidate
  if (policy.rfind("guarded", 0) == 0) {
    std::vector<const View*> videos;
    for (const auto& v : rows)
      if (&v != candidate && v.row->str("kind", "") == "video" && v.row->flag("started", false) &&
          slack_of(v, now) >= 0 && slack_of(v, now) < cost)
        videos.push_back(&v);
    std::sort(videos.begin(), videos.end(), [&](const View* a, const View* b) {
      return std::make_tuple(slack_of(*a, now), edf_key(*a)) < std::make_tuple(slack_of(*b, now), edf_key(*b));
    });
    for (const View* v : videos) {
      const auto vq = pick_quantum(*v, rows, now, quantum, costs);
      const double vc = cost_of(*v, vq.first);
      if (!vq.second && slack_of(*candidate, now) >= vc && !endangers(rows, *v, vc, now))
        return decide(*v, vq.first, "video_resume_guard", false, now);
    }
  }
  // (c) deadline conflict
  if (q.second || endangers(rows, *candidate, cost, now)) return fallback();
  return decide(*candidate, q.first, reason, false, now);
}

}  // namespace ds
