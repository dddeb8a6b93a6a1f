#include "ds/process.hpp"

#include <fcntl.h>
#include <poll.h>
#include <signal.h>
#include <spawn.h>
#include <sys/prctl.h>
#include <sys/wait.h>
#include <time.h>
#include <unistd.h>

#include <cerrno>
#include <cstring>

extern char** environ;

namespace ds {

double monotonic_seconds() {
  timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return ts.tv_sec + ts.tv_nsec * 1e-9;
}

void become_subreaper() { prctl(PR_SET_CHILD_SUBREAPER, 1, 0, 0, 0); }

WorkerProcess::WorkerProcess(const std::vector<std::string>& argv, const std::map<std::string, std::string>& env,
                             const std::string& log_path)
    : log_(log_path) {
  if (argv.empty()) throw std::invalid_argument("worker argv is empty");
  int in_pipe[2], out_pipe[2];
  if (pipe2(in_pipe, O_CLOEXEC) != 0 || pipe2(out_pipe, O_CLOEXEC) != 0)
    throw std::runtime_error(std::string("pipe: ") + std::strerror(errno));
  posix_spawn_file_actions_t fa;
  posix_spawn_file_actions_init(&fa);
  posix_spawn_file_actions_adddup2(&fa, in_pipe[0], 0);
  posix_spawn_file_actions_adddup2(&fa, out_pipe[1], 1);
  if (!log_path.empty()) posix_spawn_file_actions_addopen(&fa, 2, log_path.c_str(), O_WRONLY | O_CREAT | O_APPEND, 0644);
  posix_spawnattr_t at;
  posix_spawnattr_init(&at);
  sigset_t dflt;
  sigemptyset(&dflt);
  sigaddset(&dflt, SIGTERM);
  sigaddset(&dflt, SIGINT);
  sigaddset(&dflt, SIGPIPE);
  sigaddset(&dflt, SIGCHLD);
  sigset_t none;
  sigemptyset(&none);
  posix_spawnattr_setsigdefault(&at, &dflt);
  posix_spawnattr_setsigmask(&at, &none);
  posix_spawnattr_setpgroup(&at, 0);
  posix_spawnattr_setflags(&at, POSIX_SPAWN_SETPGROUP | POSIX_SPAWN_SETSIGDEF | POSIX_SPAWN_SETSIGMASK);
  std::vector<std::string> envs;
  for (char** e = environ; *e; ++e) {
    std::string kv(*e);
    const std::string key = kv.substr(0, kv.find('='));
    if (!env.count(key)) envs.push_back(kv);
  }
  for (const auto& kv : env) envs.push_back(kv.first + "=" + kv.second);
  std::vector<char*> cargv, cenv;
  for (const auto& a : argv) cargv.push_back(const_cast<char*>(a.c_str()));
  cargv.push_back(nullptr);
  for (const auto& e : envs) cenv.push_back(const_cast<char*>(e.c_str()));
  cenv.push_back(nullptr);
  const int rc = posix_spawnp(&pid_, cargv[0], &fa, &at, cargv.data(), cenv.data());
  posix_spawn_file_actions_destroy(&fa);
  posix_spawnattr_destroy(&at);
  close(in_pipe[0]);
  close(out_pipe[1]);
  if (rc != 0) {
    close(in_pipe[1]);
    close(out_pipe[0]);
    throw std::runtime_error("posix_spawnp " + argv[0] + ": " + std::strerror(rc));
  }
  to_child_ = in_pipe[1];
  from_child_ = out_pipe[0];
  fcntl(from_child_, F_SETFL, fcntl(from_child_, F_GETFL) | O_NONBLOCK);
}

WorkerProcess::~WorkerProcess() {
  try {
    stop(1.0);
  } catch (...) {
  }
}

bool WorkerProcess::alive() {
  if (pid_ <= 0 || stopped_) return false;
  int status = 0;
  const pid_t r = waitpid(pid_, &status, WNOHANG);
  return r == 0;
}

std::string WorkerProcess::read_line(double deadline, const std::function<void(CancelScope&)>& heartbeat) {
  double next_beat = monotonic_seconds() + 0.5;
  while (true) {
    const size_t nl = buffer_.find('\n');
    if (nl != std::string::npos) {
      std::string line = buffer_.substr(0, nl);
      buffer_.erase(0, nl + 1);
      return line;
    }
    if (buffer_.size() > kMaxMessage) throw WorkerProtocolError("worker reply exceeds 64 MiB");
    const double now = monotonic_seconds();
    if (now >= deadline) throw WorkerDeadlineExceeded("worker call deadline exceeded");
    if (heartbeat && now >= next_beat) {
      CancelScope scope;
      heartbeat(scope);
      if (scope.cancelled) throw WorkerDeadlineExceeded("worker call cancelled: " + scope.reason);
      next_beat = now + 0.5;
    }
    const double wait = std::min(deadline, next_beat) - now;
    pollfd p{from_child_, POLLIN, 0};
    const int r = poll(&p, 1, std::max(1, static_cast<int>(wait * 1000)));
    if (r < 0 && errno != EINTR) throw std::runtime_error(std::string("poll: ") + std::strerror(errno));
    if (r > 0) {
      char buf[65536];
      const ssize_t n = read(from_child_, buf, sizeof buf);
      if (n > 0) {
        buffer_.append(buf, static_cast<size_t>(n));
      } else if (n == 0) {
        throw WorkerFailure("worker closed its output (exited?)");
      } else if (errno != EAGAIN && errno != EINTR) {
        throw std::runtime_error(std::string("read: ") + std::strerror(errno));
      }
    }
  }
}

Json WorkerProcess::call_raw(const Json& envelope, double timeout_s,
                             const std::function<void(CancelScope&)>& heartbeat) {
  if (stopped_) throw WorkerFailure("worker already stopped");
  const std::string line = envelope.dump() + "\n";
  size_t off = 0;
  while (off < line.size()) {
    const ssize_t n = write(to_child_, line.data() + off, line.size() - off);
    if (n < 0) {
      if (errno == EINTR) continue;
      throw WorkerFailure(std::string("write to worker: ") + std::strerror(errno));
    }
    off += static_cast<size_t>(n);
  }
  const double deadline = monotonic_seconds() + timeout_s;
  while (true) {
    const std::string reply = read_line(deadline, heartbeat);
    Json j;
    try {
      j = Json::parse(reply);
    } catch (const JsonError& e) {
      throw WorkerProtocolError(std::string("worker wrote a non-JSON line: ") + e.what());
    }
    if (!j.is_object() || j.integer("version", 0) != 1) throw WorkerProtocolError("reply without protocol version 1");
    if (envelope.contains("id") && j.get("id") != envelope.at("id"))
      throw WorkerProtocolError("reply id " + j.get("id").dump() + " does not match request " + envelope.at("id").dump());
    return j;
  }
}

Json WorkerProcess::call(const std::string& op, const Json& request, double timeout_s,
                         const std::function<void(CancelScope&)>& heartbeat) {
  Json env = request.is_object() ? request : Json::object();
  env["version"] = 1;
  env["id"] = next_id_++;
  env["op"] = op;
  Json reply = call_raw(env, timeout_s, heartbeat);
  if (!reply.flag("ok", false)) {
    const Json& err = reply.get("error");
    throw WorkerFailure("worker op " + op + " failed: " + (err.is_string() ? err.as_string() : err.dump()));
  }
  return reply.get("result");
}

bool WorkerProcess::stop(double grace_s) {
  if (stopped_ || pid_ <= 0) return true;
  stopped_ = true;
  if (to_child_ >= 0) close(to_child_);
  to_child_ = -1;
  const pid_t pgid = pid_;
  kill(-pgid, SIGTERM);
  const double until = monotonic_seconds() + grace_s;
  int status = 0;
  bool reaped = false;
  while (monotonic_seconds() < until) {
    const pid_t r = waitpid(pid_, &status, WNOHANG);
    if (r == pid_ || (r < 0 && errno == ECHILD)) {
      reaped = true;
      break;
    }
    usleep(10000);
  }
  kill(-pgid, SIGKILL);
  if (!reaped) waitpid(pid_, &status, 0);
  // reap reparented grandchildren of the group (we are their subreaper)
  for (int i = 0; i < 200; ++i) {
    while (waitpid(-pgid, &status, WNOHANG) > 0) {
    }
    if (kill(-pgid, 0) != 0 && errno == ESRCH) break;
    usleep(5000);
  }
  if (from_child_ >= 0) close(from_child_);
  from_child_ = -1;
  return kill(-pgid, 0) != 0 && errno == ESRCH;
}

}  // namespace ds
