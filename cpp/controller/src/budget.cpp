#include "ds/budget.hpp"

#include <fcntl.h>
#include <sys/file.h>
#include <unistd.h>

#include <chrono>
#include <cmath>
#include <cstdio>
#include <fstream>
#include <sstream>

namespace ds {

namespace {
double wall_now() {
  using namespace std::chrono;
  return duration_cast<duration<double>>(system_clock::now().time_since_epoch()).count();
}
std::string dir_of(const std::string& p) {
  const auto s = p.rfind('/');
  return s == std::string::npos ? "." : p.substr(0, s);
}
}  // namespace

Budget::Budget(const std::string& path, const Json& limits, Clock clock)
    : path_(path), limits_(limits), clock_(clock ? clock : Clock(wall_now)) {
  if (!limits_.is_object() || !limits_.get("phases").is_object()) throw BudgetError("budget limits need a phases object");
  for (const auto& kv : limits_.at("phases").as_object())
    if (!(kv.second.num("gpu_seconds", -1) >= 0)) throw BudgetError("phase " + kv.first + " needs gpu_seconds >= 0");
  const std::string carry = limits_.str("carry", "none");
  if (carry != "none" && carry != "forward") throw BudgetError("carry must be none or forward");
  lock_fd_ = open((path_ + ".lock").c_str(), O_RDWR | O_CREAT | O_CLOEXEC, 0644);
  if (lock_fd_ < 0) throw BudgetError("cannot open budget lock " + path_ + ".lock");
  if (flock(lock_fd_, LOCK_EX | LOCK_NB) != 0) {
    close(lock_fd_);
    lock_fd_ = -1;
    throw BudgetError("budget ledger is locked by another controller");
  }
  load();
  verify();
}

Budget::~Budget() {
  if (lock_fd_ >= 0) {
    flock(lock_fd_, LOCK_UN);
    close(lock_fd_);
  }
}

void Budget::load() {
  std::ifstream in(path_);
  if (!in) {
    ledger_ = Json::object();
    ledger_["schema"] = "ditserve-b200.budget.v1";
    ledger_["sessions"] = Json::array();
    ledger_["poisoned"] = false;
    save();
    return;
  }
  std::stringstream ss;
  ss << in.rdbuf();
  ledger_ = Json::parse(ss.str());
}

void Budget::save() {
  const std::string tmp = path_ + ".tmp";
  {
    FILE* f = std::fopen(tmp.c_str(), "w");
    if (!f) throw BudgetError("cannot write " + tmp);
    const std::string text = ledger_.dump(1) + "\n";
    if (std::fwrite(text.data(), 1, text.size(), f) != text.size()) {
      std::fclose(f);
      throw BudgetError("short write to " + tmp);
    }
    std::fflush(f);
    fsync(fileno(f));
    std::fclose(f);
  }
  if (std::rename(tmp.c_str(), path_.c_str()) != 0) throw BudgetError("cannot rename budget ledger");
  const int d = open(dir_of(path_).c_str(), O_RDONLY | O_DIRECTORY);
  if (d >= 0) {
    fsync(d);
    close(d);
  }
}

void Budget::verify() const {
  if (ledger_.str("schema", "") != "ditserve-b200.budget.v1") throw BudgetError("unknown budget ledger schema");
  int open_sessions = 0;
  for (const auto& s : ledger_.at("sessions").as_array()) {
    const double start = s.at("start").as_double();
    const int devices = static_cast<int>(s.at("devices").as_int());
    if (devices <= 0) throw BudgetError("ledger session with no devices");
    if (s.str("state", "") == "open") {
      ++open_sessions;
      continue;
    }
    const double end = s.at("end").as_double();
    if (end < start) throw BudgetError("ledger session ends before it starts");
    const double gs = s.at("gpu_seconds").as_double();
    if (std::fabs(gs - devices * (end - start)) > 1e-6 * std::max(1.0, gs))
      throw BudgetError("ledger session GPU-seconds do not match its span");
  }
  if (open_sessions > 1) throw BudgetError("ledger has more than one open session");
}

double Budget::used(const std::string& phase, bool repair) const {
  double u = 0;
  for (const auto& s : ledger_.at("sessions").as_array()) {
    if (s.at("phase").as_string() != phase || s.flag("repair", false) != repair) continue;
    if (s.str("state", "") == "open") continue;
    u += s.at("gpu_seconds").as_double();
  }
  return u;
}

double Budget::allowance(const std::string& phase, bool repair) const {
  if (repair) return limits_.num("repair_reserve_gpu_seconds", 0.0) - [&] {
      double u = 0;
      for (const auto& kv : limits_.at("phases").as_object()) u += used(kv.first, true);
      return u;
    }();
  const Json& p = limits_.at("phases").get(phase);
  if (p.is_null()) throw BudgetError("no budget for phase " + phase);
  double left = p.at("gpu_seconds").as_double() - used(phase, false);
  if (limits_.str("carry", "none") == "forward") {
    for (const auto& kv : limits_.at("phases").as_object()) {
      if (kv.first == phase) break;  // phases carry into later ones (map order = name order)
      left += std::max(0.0, kv.second.at("gpu_seconds").as_double() - used(kv.first, false));
    }
  }
  return left;
}

std::string Budget::begin(const std::string& identity, int devices, const std::string& phase, double watchdog_s,
                          bool repair) {
  if (!open_.is_null()) throw BudgetError("a budget session is already open");
  if (poisoned() && !repair) throw BudgetError("budget ledger is poisoned by an unverified cleanup; run a repair");
  if (devices <= 0) throw BudgetError("devices must be positive");
  const double left = allowance(phase, repair);
  if (left <= 0) throw BudgetError("no GPU-seconds left for phase " + phase);
  const double start = clock_();
  Json s = Json::object();
  s["id"] = identity + "#" + std::to_string(ledger_.at("sessions").size());
  s["identity"] = identity;
  s["phase"] = phase;
  s["devices"] = devices;
  s["start"] = start;
  s["repair"] = repair;
  s["state"] = "open";
  s["deadline"] = start + std::min(watchdog_s > 0 ? watchdog_s : 1e18, left / devices);
  ledger_["sessions"].push_back(s);
  save();
  open_ = s;
  return s.at("id").as_string();
}

double Budget::deadline() const {
  if (open_.is_null()) throw BudgetError("no open budget session");
  return open_.at("deadline").as_double();
}

void Budget::check() const {
  if (clock_() > deadline()) throw BudgetError("budget deadline passed for session " + open_.at("id").as_string());
}

Json Budget::finish(const std::string& status, bool cleanup_verified) {
  if (open_.is_null()) throw BudgetError("no open budget session");
  auto& sessions = ledger_["sessions"].as_array();
  Json& s = sessions.back();
  const double end = clock_();
  s["end"] = end;
  s["gpu_seconds"] = s.at("devices").as_int() * (end - s.at("start").as_double());
  s["status"] = status;
  s["cleanup_verified"] = cleanup_verified;
  s["state"] = "settled";
  if (!cleanup_verified) ledger_["poisoned"] = true;
  else if (s.flag("repair", false)) ledger_["poisoned"] = false;
  save();
  Json out = s;
  open_ = Json();
  return out;
}

}  // namespace ds
