// GPU-second budget ledger.
//
// One JSON ledger per study root, guarded by flock on a sibling lock file and
// rewritten atomically (write temp, fsync, rename, fsync dir).  Limits are per
// phase in GPU-seconds with carry "none" (unused time is lost) or "forward"
// (unused time of earlier phases adds to this one) plus a repair reserve that
// only `--repair` sessions draw from.  begin() opens a session (devices,
// watchdog); deadline() is the monotonic instant its allowance runs out;
// finish() settles it and, unless cleanup was verified, poisons the ledger so
// no new session starts until a repair settles it.  History is re-validated on
// every open.  The clock is injectable for tests.
// Reference semantics: src/ditserve/control/budget.cpp:71-276.
#pragma once
#include <functional>
#include <string>

#include "ds/json.hpp"

namespace ds {

class BudgetError : public std::runtime_error {
 public:
  using std::runtime_error::runtime_error;
};

class Budget {
 public:
  using Clock = std::function<double()>;  // wall seconds
  Budget(const std::string& path, const Json& limits, Clock clock = {});
  ~Budget();
  Budget(const Budget&) = delete;
  Budget& operator=(const Budget&) = delete;

  double allowance(const std::string& phase, bool repair = false) const;  // GPU-seconds left
  // returns the session id
  std::string begin(const std::string& identity, int devices, const std::string& phase, double watchdog_s,
                    bool repair = false);
  double deadline() const;  // wall-clock second at which the open session must end
  void check() const;       // throws BudgetError past the deadline
  Json finish(const std::string& status, bool cleanup_verified);
  const Json& ledger() const { return ledger_; }
  bool poisoned() const { return ledger_.flag("poisoned", false); }

 private:
  void load();
  void save();
  void verify() const;
  double used(const std::string& phase, bool repair) const;
  std::string path_;
  Json limits_;
  Clock clock_;
  int lock_fd_ = -1;
  Json ledger_;
  Json open_;  // current session
};

}  // namespace ds
