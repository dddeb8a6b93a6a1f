// Worker process supervision and the JSON-lines RPC.
//
// A worker is spawned with posix_spawnp into its own process group (the
// controller is a child subreaper, so grandchildren cannot escape), stdin and
// stdout are pipes, stderr goes to a per-worker log file.  call() writes one
// request line {"version":1,"id":N,"op":...} and waits, with poll() against an
// absolute monotonic deadline, for the reply line with the same id; a
// heartbeat callback runs every 0.5 s while waiting and may cancel.  Replies
// are capped at 64 MiB.  stop() sends SIGTERM to the group, SIGKILL after the
// grace period, reaps the leader and verifies the group is gone.
// Reference semantics: src/ditserve/runtime/process.cpp:182-370.
#pragma once
#include <sys/types.h>

#include <functional>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

#include "ds/json.hpp"

namespace ds {

double monotonic_seconds();

class WorkerDeadlineExceeded : public std::runtime_error {
 public:
  using std::runtime_error::runtime_error;
};
class WorkerFailure : public std::runtime_error {  // the worker answered ok=false or died
 public:
  using std::runtime_error::runtime_error;
};
class WorkerProtocolError : public std::runtime_error {
 public:
  using std::runtime_error::runtime_error;
};

struct CancelScope {
  bool cancelled = false;
  std::string reason;
  void cancel(const std::string& why) {
    cancelled = true;
    reason = why;
  }
};

class WorkerProcess {
 public:
  static constexpr size_t kMaxMessage = 64u << 20;
  WorkerProcess(const std::vector<std::string>& argv, const std::map<std::string, std::string>& env,
                const std::string& log_path);
  ~WorkerProcess();
  WorkerProcess(const WorkerProcess&) = delete;
  WorkerProcess& operator=(const WorkerProcess&) = delete;

  // op fields go in `request`; returns the reply's "result" (throws on ok=false)
  Json call(const std::string& op, const Json& request, double timeout_s,
            const std::function<void(CancelScope&)>& heartbeat = {});
  // raw envelope exchange (tests)
  Json call_raw(const Json& envelope, double timeout_s, const std::function<void(CancelScope&)>& heartbeat = {});
  bool alive();
  bool stop(double grace_s = 2.0);  // true when the whole process group is verified gone
  pid_t pid() const { return pid_; }
  const std::string& log_path() const { return log_; }

 private:
  std::string read_line(double deadline, const std::function<void(CancelScope&)>& heartbeat);
  pid_t pid_ = -1;
  int to_child_ = -1, from_child_ = -1;
  long long next_id_ = 1;
  std::string buffer_;
  std::string log_;
  bool stopped_ = false;
};

void become_subreaper();

}  // namespace ds
