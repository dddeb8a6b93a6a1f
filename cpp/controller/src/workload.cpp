#include "ds/workload.hpp"

#include <algorithm>
#include <cmath>
#include <set>
#include <stdexcept>

#include "ds/rng.hpp"

namespace ds {

double quantile(std::vector<double> v, double q) {
  if (v.empty()) return 0.0;
  std::sort(v.begin(), v.end());
  // linear interpolation between closest ranks
  const double pos = q * (v.size() - 1);
  const size_t lo = static_cast<size_t>(std::floor(pos));
  const size_t hi = std::min(v.size() - 1, lo + 1);
  return v[lo] + (pos - lo) * (v[hi] - v[lo]);
}

static double positive(const Json& j, const std::string& key, double dflt) {
  const double v = j.num(key, dflt);
  if (!std::isfinite(v) || v <= 0) throw std::invalid_argument(key + " must be positive");
  return v;
}

Json study_workload(const Json& phase) {
  Json rows = phase.get("workload").is_null() ? Json::array() : phase.at("workload");
  if (!rows.is_array()) throw std::invalid_argument("workload must be an array");
  if (rows.empty() && phase.contains("generator")) {
    const Json& g = phase.at("generator");
    const long long seed = g.integer("seed", 7);
    Random arrivals(static_cast<uint64_t>(seed));
    Random content(static_cast<uint64_t>(seed) ^ 0x9E3779B97F4A7C15ull);
    const int count = static_cast<int>(g.integer("count", 8));
    if (count < 0 || count > 1000000) throw std::invalid_argument("count out of range");
    const std::string pattern = g.str("pattern", "offline_all");
    if (pattern != "offline_all" && pattern != "steady" && pattern != "poisson" && pattern != "bursty" &&
        pattern != "gamma")
      throw std::invalid_argument("unknown arrival pattern " + pattern);
    double rate = g.contains("rate_rpm") ? positive(g, "rate_rpm", 1) / 60.0 : positive(g, "rate_rps", 1);
    const double cv = positive(g, "cv", 2.0);
    const double period = positive(g, "burst_period_ms", 1000.0);
    const double active = positive(g, "burst_active_fraction", 0.2);
    if (active > 1) throw std::invalid_argument("burst_active_fraction must be <= 1");
    const Json classes = g.get("classes").is_null() ? Json::array() : g.at("classes");
    double total_w = 0;
    for (const auto& c : classes.as_array()) total_w += positive(c, "weight", 1.0);
    double t = 0;
    for (int i = 0; i < count; ++i) {
      if (i > 0) {
        if (pattern == "steady") t += 1000.0 / rate;
        else if (pattern == "gamma") t += arrivals.gamma(1.0 / (cv * cv), cv * cv) * 1000.0 / rate;
        else if (pattern == "poisson") t += arrivals.exponential(rate / 1000.0);
        else if (pattern == "bursty") t += arrivals.exponential(rate / 1000.0 / active);
      }
      double arrival = 0;
      if (pattern == "bursty") arrival = std::floor(t / (period * active)) * period + std::fmod(t, period * active);
      else if (pattern != "offline_all") arrival = t;
      Json row = Json::object();
      row["request_id"] = "r" + std::to_string(i);
      row["arrival_ms"] = arrival;
      Json spec = Json::object();
      if (classes.empty()) {
        spec = g.get("spec").is_null() ? Json::object() : g.at("spec");
        row["service_ms"] = g.num("service_ms", 100.0);
        row["slo_ms"] = g.num("slo_ms", 250.0);
      } else {
        double pick = content.uniform() * total_w;
        size_t k = 0;
        for (; k + 1 < classes.size(); ++k) {
          pick -= positive(classes[k], "weight", 1.0);
          if (pick < 0) break;
        }
        const Json& c = classes[k];
        spec = c.get("spec").is_null() ? Json::object() : c.at("spec");
        const double service = positive(c, "service_ms", 100.0);
        row["service_ms"] = service;
        double slo;
        if (c.contains("slo_ms")) {
          slo = positive(c, "slo_ms", 1.0);
        } else if (c.contains("slo_scale_range")) {
          const auto& r = c.at("slo_scale_range");
          slo = service * content.uniform(r[0].as_double(), r[1].as_double());
        } else {
          slo = service * positive(c, "slo_scale", 2.5);
        }
        row["slo_ms"] = slo;
        row["kind"] = c.at("kind");
        row["class"] = c.at("class");
        if (c.contains("worker")) row["worker"] = c.at("worker");
      }
      spec["seed"] = static_cast<long long>(content.below(1ull << 31));
      row["spec"] = spec;
      rows.push_back(row);
    }
  }
  std::set<std::string> ids;
  for (size_t i = 0; i < rows.size(); ++i) {
    Json& row = rows[i];
    if (!row.contains("request_id")) row["request_id"] = "r" + std::to_string(i);
    const std::string id = row.at("request_id").as_string();
    if (id.empty() || !ids.insert(id).second) throw std::invalid_argument("duplicate or empty request_id");
    row["arrival_ms"] = row.num("arrival_ms", 0.0);
    row["service_ms"] = row.num("service_ms", phase.num("service_ms", 100.0));
    row["slo_ms"] = row.num("slo_ms", row.at("service_ms").as_double() * 2.5);
    row["deadline_ms"] = row.num("deadline_ms", row.at("arrival_ms").as_double() + row.at("slo_ms").as_double());
    if (row.at("deadline_ms").as_double() < row.at("arrival_ms").as_double())
      throw std::invalid_argument("deadline before arrival for " + id);
    if (!row.contains("spec")) row["spec"] = phase.get("spec").is_null() ? Json::object() : phase.at("spec");
    row["spec"]["request_id"] = id;
    if (!row.contains("worker")) row["worker"] = phase.str("worker", "model");
    if (!row.contains("kind")) row["kind"] = phase.str("request_kind", "video");
    if (!row.contains("class")) row["class"] = phase.str("class", row.at("kind").as_string());
    row["status"] = "pending";
  }
  std::set<std::string> before;
  for (const auto& row : rows.as_array()) {
    if (row.contains("after") && !before.count(row.at("after").as_string()))
      throw std::invalid_argument("a predecessor must precede its request in the trace");
    before.insert(row.at("request_id").as_string());
  }
  return rows;
}

static Json summarise(const Json& rows, const std::string* kind) {
  size_t total = 0, done = 0, ontime = 0, failed = 0, censored = 0, not_executed = 0;
  double exposure = 0;
  std::vector<double> lat;
  for (const auto& r : rows.as_array()) {
    if (kind && r.str("kind", "") != *kind) continue;
    ++total;
    const std::string st = r.str("status", "pending");
    const double arrival = r.num("arrival_ms", 0.0);
    if (st == "done" || st == "ok") {
      ++done;
      const double fin = r.at("finish_ms").as_double();
      lat.push_back(fin - arrival);
      if (fin <= r.num("deadline_ms", 1e300)) ++ontime;
      exposure = std::max(exposure, fin);
    } else if (st == "failed") {
      ++failed;
    } else if (st == "censored") {
      ++censored;
    } else {
      ++not_executed;
    }
    exposure = std::max(exposure, r.num("observation_ms", 0.0));
  }
  Json s = Json::object();
  s["requests"] = static_cast<long long>(total);
  s["completed"] = static_cast<long long>(done);
  s["on_time"] = static_cast<long long>(ontime);
  s["failed"] = static_cast<long long>(failed);
  s["censored"] = static_cast<long long>(censored);
  s["not_executed"] = static_cast<long long>(not_executed);
  s["slo_attainment"] = total ? static_cast<double>(ontime) / total : 0.0;
  s["exposure_ms"] = exposure;
  s["goodput_rps"] = exposure > 0 ? ontime / (exposure / 1000.0) : 0.0;
  s["goodput_rpm"] = exposure > 0 ? ontime / (exposure / 60000.0) : 0.0;
  s["latency_p50_ms"] = quantile(lat, 0.50);
  s["latency_p95_ms"] = quantile(lat, 0.95);
  s["latency_p99_ms"] = quantile(lat, 0.99);
  s["latency_mean_ms"] = lat.empty() ? 0.0 : [&] {
    double a = 0;
    for (double v : lat) a += v;
    return a / lat.size();
  }();
  return s;
}

Json request_summary(const Json& rows) {
  if (!rows.is_array()) throw std::invalid_argument("metric rows must be an array");
  Json s = summarise(rows, nullptr);
  Json kinds = Json::object();
  std::set<std::string> names;
  for (const auto& r : rows.as_array()) names.insert(r.str("kind", "video"));
  for (const auto& k : names) kinds[k] = summarise(rows, &k);
  s["kinds"] = kinds;
  return s;
}

Json kind_summary(const Json& rows, const std::string& kind) { return summarise(rows, &kind); }

// ---------------------------------------------------------------------------------------
static std::vector<std::string> pointer_tokens(const std::string& p) {
  std::vector<std::string> out;
  if (p.empty()) return out;
  if (p[0] != '/') throw std::invalid_argument("JSON pointer must start with '/': " + p);
  size_t i = 1;
  while (true) {
    size_t j = p.find('/', i);
    std::string tok = p.substr(i, j == std::string::npos ? std::string::npos : j - i);
    std::string dec;
    for (size_t k = 0; k < tok.size(); ++k) {
      if (tok[k] == '~' && k + 1 < tok.size() && (tok[k + 1] == '0' || tok[k + 1] == '1')) {
        dec.push_back(tok[k + 1] == '0' ? '~' : '/');
        ++k;
      } else {
        dec.push_back(tok[k]);
      }
    }
    out.push_back(dec);
    if (j == std::string::npos) break;
    i = j + 1;
  }
  return out;
}

const Json* json_pointer_get(const Json& doc, const std::string& pointer) {
  const Json* cur = &doc;
  for (const auto& tok : pointer_tokens(pointer)) {
    if (cur->is_object()) {
      if (!cur->contains(tok)) return nullptr;
      cur = &cur->at(tok);
    } else if (cur->is_array()) {
      if (tok.empty() || tok.find_first_not_of("0123456789") != std::string::npos) return nullptr;
      const size_t idx = std::stoul(tok);
      if (idx >= cur->size()) return nullptr;
      cur = &cur->at(idx);
    } else {
      return nullptr;
    }
  }
  return cur;
}

void json_pointer_set(Json& doc, const std::string& pointer, const Json& value) {
  auto toks = pointer_tokens(pointer);
  if (toks.empty()) {
    doc = value;
    return;
  }
  Json* cur = &doc;
  for (size_t i = 0; i + 1 < toks.size(); ++i) {
    if (cur->is_array()) cur = &cur->at(std::stoul(toks[i]));
    else cur = &(*cur)[toks[i]];
  }
  if (cur->is_array()) cur->at(std::stoul(toks.back())) = value;
  else (*cur)[toks.back()] = value;
}

Json evaluate_gates(const Json& evidence, const Json& rules) {
  Json out = Json::object();
  Json results = Json::array();
  bool pass = true;
  for (const auto& r : rules.as_array()) {
    const std::string ptr = r.at("pointer").as_string();
    const std::string op = r.str("op", ">=");
    const Json& want = r.at("value");
    const Json* got = json_pointer_get(evidence, ptr);
    bool ok = false;
    if (got != nullptr) {
      if (got->is_number() && want.is_number()) {
        const double a = got->as_double(), b = want.as_double();
        if (op == "<") ok = a < b;
        else if (op == "<=") ok = a <= b;
        else if (op == ">") ok = a > b;
        else if (op == ">=") ok = a >= b;
        else if (op == "==") ok = a == b;
        else if (op == "!=") ok = a != b;
        else throw std::invalid_argument("unknown gate op " + op);
      } else if (op == "==") {
        ok = *got == want;
      } else if (op == "!=") {
        ok = *got != want;
      } else {
        throw std::invalid_argument("gate " + ptr + ": ordered comparison needs numbers");
      }
    }
    Json row = Json::object();
    row["pointer"] = ptr;
    row["op"] = op;
    row["value"] = want;
    row["observed"] = got ? *got : Json();
    row["pass"] = ok;
    results.push_back(row);
    pass = pass && ok;
  }
  out["pass"] = pass;
  out["results"] = results;
  return out;
}

Json expand_matrix(const Json& phase) {
  Json cells = Json::array();
  const Json& m = phase.get("matrix");
  if (m.is_null()) {
    cells.push_back(phase);
    return cells;
  }
  // two spellings: {"axes": [{"pointer": p, "values": [...]}, ...]} or {"/pointer": [...], ...}
  Json axes_json = Json::array();
  if (m.contains("axes")) {
    axes_json = m.at("axes");
  } else {
    for (const auto& kv : m.as_object()) {
      Json a = Json::object();
      a["pointer"] = kv.first;
      a["values"] = kv.second;
      axes_json.push_back(a);
    }
  }
  const auto& axes = axes_json.as_array();
  size_t total = 1;
  for (const auto& a : axes) {
    const size_t k = a.at("values").size();
    if (k == 0) throw std::invalid_argument("matrix axis without values");
    total *= k;
    if (total > 10000) throw std::invalid_argument("matrix exceeds 10000 cells");
  }
  for (size_t idx = 0; idx < total; ++idx) {
    Json cell = phase;
    cell.as_object().erase("matrix");
    Json coords = Json::object();
    size_t rem = idx;
    for (size_t a = axes.size(); a-- > 0;) {
      const auto& vals = axes[a].at("values");
      const size_t k = rem % vals.size();
      rem /= vals.size();
      json_pointer_set(cell, axes[a].at("pointer").as_string(), vals[k]);
      coords[axes[a].at("pointer").as_string()] = vals[k];
    }
    cell["cell"] = static_cast<long long>(idx);
    cell["coordinates"] = coords;
    cells.push_back(cell);
  }
  return cells;
}

}  // namespace ds
