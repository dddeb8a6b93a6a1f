#include "ds/study.hpp"

#include <dirent.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <fstream>
#include <functional>
#include <future>
#include <map>
#include <memory>
#include <mutex>
#include <set>
#include <sstream>
#include <stdexcept>
#include <thread>

#include "ds/budget.hpp"
#include "ds/cost.hpp"
#include "ds/dispatch.hpp"
#include "ds/planner.hpp"
#include "ds/policy.hpp"
#include "ds/process.hpp"
#include "ds/sim.hpp"
#include "ds/workload.hpp"

namespace ds {
namespace {

void mkdirs(const std::string& path) {
  std::string cur;
  std::stringstream ss(path);
  std::string part;
  if (!path.empty() && path[0] == '/') cur = "/";
  while (std::getline(ss, part, '/')) {
    if (part.empty()) continue;
    cur += part + "/";
    mkdir(cur.c_str(), 0755);
  }
}

bool exists(const std::string& p) {
  struct stat st;
  return stat(p.c_str(), &st) == 0;
}

std::string read_file(const std::string& p) {
  std::ifstream in(p);
  if (!in) throw std::runtime_error("cannot read " + p);
  std::stringstream ss;
  ss << in.rdbuf();
  return ss.str();
}

void write_atomic(const std::string& p, const std::string& text) {
  const std::string tmp = p + ".tmp";
  {
    std::ofstream out(tmp);
    if (!out) throw std::runtime_error("cannot write " + tmp);
    out << text;
    out.flush();
  }
  if (std::rename(tmp.c_str(), p.c_str()) != 0) throw std::runtime_error("cannot rename " + tmp);
}

std::string fnv1a(const std::string& s) {
  uint64_t h = 1469598103934665603ull;
  for (unsigned char c : s) {
    h ^= c;
    h *= 1099511628211ull;
  }
  char buf[20];
  std::snprintf(buf, sizeof buf, "%016llx", static_cast<unsigned long long>(h));
  return buf;
}

double now_ms_since(double t0) { return (monotonic_seconds() - t0) * 1000.0; }

// FNV-1a over a file's bytes, folded into `h`
uint64_t hash_file(const std::string& path, uint64_t h) {
  std::ifstream in(path, std::ios::binary);
  char buf[1 << 16];
  while (in) {
    in.read(buf, sizeof buf);
    for (std::streamsize i = 0; i < in.gcount(); ++i) {
      h ^= static_cast<unsigned char>(buf[i]);
      h *= 1099511628211ull;
    }
  }
  return h;
}

void list_code(const std::string& dir, std::vector<std::string>& out) {
  DIR* d = opendir(dir.c_str());
  if (!d) return;
  while (dirent* e = readdir(d)) {
    const std::string n = e->d_name;
    if (n == "." || n == ".." || n == "__pycache__") continue;
    const std::string p = dir + "/" + n;
    struct stat st;
    if (stat(p.c_str(), &st) != 0) continue;
    if (S_ISDIR(st.st_mode)) {
      list_code(p, out);
      continue;
    }
    for (const char* ext : {".py", ".cu", ".cuh", ".cpp", ".h", ".so"}) {
      const std::string x(ext);
      if (n.size() > x.size() && n.compare(n.size() - x.size(), x.size(), x) == 0) {
        out.push_back(p);
        break;
      }
    }
  }
  closedir(d);
}

// the code a run depends on: this controller binary and the worker package's sources and
// compiled extension; a resumed run must present the same hashes
Json code_identity(const StudyOptions& opt) {
  Json c = Json::object();
  char exe[4096] = {0};
  const ssize_t n = readlink("/proc/self/exe", exe, sizeof exe - 1);
  char hex[20];
  if (n > 0) {
    std::snprintf(hex, sizeof hex, "%016llx",
                  static_cast<unsigned long long>(hash_file(std::string(exe, n), 1469598103934665603ull)));
    c["controller"] = hex;
  }
  if (!opt.package_root.empty()) {
    std::vector<std::string> files;
    list_code(opt.package_root + "/ditserve_b200", files);
    std::sort(files.begin(), files.end());
    uint64_t h = 1469598103934665603ull;
    for (const auto& f : files) {
      for (unsigned char ch : f.substr(opt.package_root.size())) {
        h ^= ch;
        h *= 1099511628211ull;
      }
      h = hash_file(f, h);
    }
    std::snprintf(hex, sizeof hex, "%016llx", static_cast<unsigned long long>(h));
    c["worker_package"] = hex;
    c["files"] = static_cast<long long>(files.size());
  }
  return c;
}

// one worker process with serialised calls
struct Worker {
  std::unique_ptr<WorkerProcess> proc;
  std::mutex mu;
  std::string name;
  Json call(const std::string& op, const Json& req, double timeout_s = 600) {
    std::lock_guard<std::mutex> lock(mu);
    return proc->call(op, req, timeout_s);
  }
};

std::unique_ptr<Worker> spawn_worker(const Json& def, const StudyOptions& opt, const std::string& log,
                                     const std::string& gpu) {
  const std::string backend = def.at("backend").as_string();
  const bool gpu_backend = backend == "wan" || backend == "sd35";
  if (gpu_backend && !opt.allow_gpu) throw std::runtime_error("backend " + backend + " needs --allow-gpu");
  const std::string config = (def.get("config").is_null() ? Json::object() : def.at("config")).dump();
  std::vector<std::string> argv = {def.str("python", opt.python), "-m", "ditserve_b200.runtime.worker",
                                   "--backend", backend, "--config", config};
  std::map<std::string, std::string> env;
  if (!opt.package_root.empty()) env["PYTHONPATH"] = opt.package_root;
  if (def.contains("remote")) {
    // a worker on another node: the local process is the bridge proxy (worker protocol on
    // stdin/stdout, relayed to the node's daemon); the remote worker gets remote_env
    argv = {def.str("python", opt.python), "-m", "ditserve_b200.runtime.remote_bridge", "proxy", "--connect",
            def.at("remote").as_string(), "--backend", backend, "--config", config};
    if (def.contains("remote_env"))
      for (const auto& [k, v] : def.at("remote_env").as_object()) {
        argv.push_back("--env");
        argv.push_back(k + "=" + (v.is_string() ? v.as_string() : v.dump()));
      }
    env["CUDA_VISIBLE_DEVICES"] = "";
  } else if (gpu == "all") {
    // every GPU visible (world members address their peers' memory); device chosen in config
  } else if (!gpu.empty()) {
    env["CUDA_VISIBLE_DEVICES"] = gpu;
  } else if (!gpu_backend) {
    env["CUDA_VISIBLE_DEVICES"] = "";
  }
  auto w = std::make_unique<Worker>();
  w->name = backend;
  w->proc = std::make_unique<WorkerProcess>(argv, env, log);
  w->proc->call("hello", Json::object(), 120);
  return w;
}

// ---------------------------------------------------------------------------------------
Json run_operations(const Json& phase, Worker& w) {
  Json results = Json::array();
  for (const auto& step : phase.at("operations").as_array()) {
    Json req = step;
    const std::string op = req.at("op").as_string();
    req.as_object().erase("op");
    const bool expect_fail = req.flag("expect_failure", false);
    req.as_object().erase("expect_failure");
    Json row = Json::object();
    row["op"] = op;
    try {
      row["result"] = w.call(op, req);
      row["ok"] = true;
      if (expect_fail) throw std::runtime_error("operation " + op + " was expected to fail");
    } catch (const WorkerFailure& e) {
      row["ok"] = false;
      row["error"] = e.what();
      if (!expect_fail) throw;
    }
    results.push_back(row);
  }
  Json out = Json::object();
  out["operations"] = results;
  return out;
}

Json run_online(const Json& phase, Worker& w) {
  Json rows = study_workload(phase);
  const std::string policy = phase.str("policy", "edf");
  if (!is_online_policy(policy)) throw std::invalid_argument("unknown online policy " + policy);
  const Json default_quantum = phase.contains("quantum_steps") ? phase.at("quantum_steps") : Json(1);
  const Json costs = phase.get("costs").is_null() ? Json::object() : phase.at("costs");
  std::map<std::string, Json*> by_id;
  for (auto& r : rows.as_array()) by_id[r.at("request_id").as_string()] = &r;
  const double t0 = monotonic_seconds();
  std::set<std::string> prepared, done;
  std::map<std::string, double> remaining, ready_since;
  std::map<std::string, int> steps_left;
  std::string active;
  Json decisions = Json::array();
  while (done.size() < rows.size()) {
    const double now = now_ms_since(t0);
    Json visible = Json::array();
    double next_arrival = 1e300;
    for (const auto& r : rows.as_array()) {
      const std::string id = r.at("request_id").as_string();
      if (done.count(id)) continue;
      const double arrival = r.at("arrival_ms").as_double();
      if (arrival > now) {
        next_arrival = std::min(next_arrival, arrival);
        continue;
      }
      const double service = r.at("service_ms").as_double();
      const int steps = static_cast<int>(r.at("spec").integer("steps", 1));
      const int left = steps_left.count(id) ? steps_left[id] : steps;
      const double per_step = service / std::max(1, steps);
      Json v = Json::object();
      v["request_id"] = id;
      v["kind"] = r.str("kind", "video");
      v["status"] = "pending";
      v["arrival_ms"] = arrival;
      v["deadline_ms"] = r.at("deadline_ms");
      v["remaining_ms"] = remaining.count(id) ? remaining[id] : service;
      v["service_ms"] = service;
      v["ready_since_ms"] = std::min(now, ready_since.count(id) ? ready_since[id] : arrival);
      v["action"] = v.at("kind").as_string() == "image" ? "image" : "denoise";
      v["started"] = prepared.count(id) > 0;
      Json table = Json::object();
      for (int q : {1, 2, 4, 8}) table[std::to_string(q)] = per_step * std::min(q, left);
      table["step"] = per_step;
      v["action_ms_by_quantum"] = table;
      // session view of the same request (one stage)
      v["ready"] = true;
      v["release_ms"] = arrival;
      v["stage_deadline_ms"] = r.at("deadline_ms");
      v["remaining_total_ms"] = v.at("remaining_ms");
      visible.push_back(v);
    }
    if (visible.empty()) {
      std::this_thread::sleep_for(std::chrono::duration<double, std::milli>(std::max(0.0, next_arrival - now)));
      continue;
    }
    const Json d = select_online(visible, now, policy, active, default_quantum, costs);
    if (d.at("request_id").is_null()) {
      std::this_thread::sleep_for(std::chrono::milliseconds(1));
      continue;
    }
    if (decisions.size() < 4096) {
      Json rec = d;
      rec["t_ms"] = now;
      decisions.push_back(rec);
    }
    const std::string id = d.at("request_id").as_string();
    const Json q = d.at("quantum");
    const int steps_now = q.is_number() ? std::max(1, static_cast<int>(q.as_int())) : 1;
    active = id;
    Json& row = *by_id[id];
    if (!prepared.count(id)) {
      Json req = Json::object();
      req["state_id"] = id;
      req["spec"] = row.at("spec");
      w.call("prepare", req);
      prepared.insert(id);
      if (!row.contains("start_ms")) row["start_ms"] = now_ms_since(t0);
    }
    Json adv = Json::object();
    adv["state_id"] = id;
    adv["steps"] = steps_now;
    Json res = w.call("advance", adv);
    const Json& prog = res.at("progress");
    const double total = prog.at("steps").as_double();
    const double frac = total > 0 ? prog.at("step").as_double() / total : 1;
    remaining[id] = row.at("service_ms").as_double() * (1 - frac);
    steps_left[id] = static_cast<int>(total - prog.at("step").as_double());
    ready_since[id] = now_ms_since(t0);
    if (prog.flag("done", false)) {
      Json fin = Json::object();
      fin["state_id"] = id;
      fin["output_mode"] = phase.str("output_mode", "digest");
      Json art = w.call("finish", fin);
      Json rel = Json::object();
      rel["state_id"] = id;
      w.call("release", rel);
      row["status"] = "done";
      row["finish_ms"] = now_ms_since(t0);
      if (art.contains("value")) row["digest"] = art.at("value");
      done.insert(id);
      active.clear();
    }
  }
  for (auto& r : rows.as_array()) r["observation_ms"] = now_ms_since(t0);
  Json out = Json::object();
  out["rows"] = rows;
  out["summary"] = request_summary(rows);
  out["decisions"] = decisions;
  return out;
}

// ---------------------------------------------------------------------------------------
// Multi-GPU cluster executor.  Each GPU slot has a video worker and (optionally) an image
// worker.  With `distributed: true` the video workers form one torch.distributed world
// (NCCL on GPUs) and every member of a request's group runs the quantum under the
// assigned CFG x SP layout; otherwise the group's leader runs it alone.  A request's state
// is tracked per worker: `fresh` copies are current, `stale` ones are outdated and get
// released.  When a group gains members the state reaches them by `sp_transport`:
// "collective" (a regroup broadcast over the new group: peer-memory put kernels or NCCL)
// or "export" (host-staged continuation packets).  A request inside a solver step keeps
// its group and form until the step ends.  Reference: study.cpp:781-2206 (cluster()).
struct Live {
  std::string id, kind, klass, status = "future";
  Json row;
  int steps_total = 1, steps_done = 0, blocks_done = 0;
  std::vector<int> group, last_group;
  std::string form, last_form;
  std::set<int> fresh, stale;
  bool prepared = false;
  double quantum_started = 0;
  bool rung = false;
  bool fold_eligible = false;  // the worker reports that the next step may run CFG-folded
  int decode_done = 0;       // decoded chunks (planner unit)
  std::string decode_ticket; // worker ticket of a chunked decode in progress
  int decode_gpu = -1;       // the worker that holds it
};

Json ints_json(const std::vector<int>& v) {
  Json a = Json::array();
  for (int x : v) a.push_back(x);
  return a;
}

// a failure that is a consequence of another member's failure (its peer stopped answering, a
// collective timed out waiting for it, or the pipe to a dead worker broke)
bool secondary_failure(const std::string& m) {
  for (const char* k : {"deadline", "closed its output", "write to worker", "already stopped", "timed out",
                        "Timeout", "Connection reset", "Broken pipe", "peer flag wait"})
    if (m.find(k) != std::string::npos) return true;
  return false;
}

// run fn(g) for every g in gs concurrently (one thread per extra member); when members fail,
// the primary failure is rethrown in preference to the secondary ones it caused
std::vector<Json> fan_out(const std::vector<int>& gs, const std::function<Json(int)>& fn) {
  std::vector<std::future<Json>> fs;
  for (size_t i = 1; i < gs.size(); ++i) fs.push_back(std::async(std::launch::async, fn, gs[i]));
  std::vector<Json> out;
  std::vector<std::pair<std::exception_ptr, std::string>> errs;
  auto note = [&](std::exception_ptr e) {
    std::string m;
    try {
      std::rethrow_exception(e);
    } catch (const std::exception& x) {
      m = x.what();
    } catch (...) {
      m = "unknown error";
    }
    errs.push_back({e, m});
  };
  try {
    out.push_back(fn(gs[0]));
  } catch (...) {
    note(std::current_exception());
  }
  for (auto& f : fs) {
    try {
      out.push_back(f.get());
    } catch (...) {
      note(std::current_exception());
    }
  }
  if (!errs.empty()) {
    for (const auto& e : errs)
      if (!secondary_failure(e.second)) std::rethrow_exception(e.first);
    std::rethrow_exception(errs.front().first);
  }
  return out;
}

Json run_cluster(const Json& phase, const StudyOptions& opt, const std::string& run_dir, const Json& workers_def) {
  const int gpus = static_cast<int>(phase.integer("gpus", 8));
  const std::string policy = phase.str("policy", "ditserve");
  Json options = phase.get("options").is_null() ? Json::object() : phase.at("options");
  const ClusterCost cost(phase.get("profile").is_null() ? synthetic_profile() : phase.at("profile"));
  std::string vname = phase.str("worker", "model"), iname = vname;
  if (phase.contains("workers")) {
    vname = phase.at("workers").str("video", vname);
    iname = phase.at("workers").str("image", vname);
  }
  const Json& vdef = workers_def.at(vname);
  const Json& idef = workers_def.at(iname);
  const bool distributed = phase.flag("distributed", false);
  const std::string transport = phase.str("sp_transport", distributed ? "collective" : "export");
  if (transport != "collective" && transport != "export")
    throw std::invalid_argument("sp_transport must be collective or export");
  if (transport == "collective" && !distributed)
    throw std::invalid_argument("sp_transport collective needs distributed: true");
  // remote_slots: {"<slot>": {"address": "host:port", "device": "<GPU index on that node>"}}
  // puts a slot's workers on another node behind the bridge; state reaches them by host-staged
  // continuation packets, so the peer-memory world (one node) is not available with them
  const Json remote_slots = phase.get("remote_slots").is_null() ? Json::object() : phase.at("remote_slots");
  if (!remote_slots.is_object()) throw std::invalid_argument("remote_slots must be an object");
  std::set<int> remote;
  for (const auto& [k, v] : remote_slots.as_object()) {
    const int g = std::stoi(k);
    if (g < 0 || g >= gpus) throw std::invalid_argument("remote slot " + k + " outside the phase's GPUs");
    if (!v.is_object() || !v.contains("address")) throw std::invalid_argument("remote slot " + k + " needs an address");
    remote.insert(g);
  }
  // nodes: this node's slots and each remote address's slots.  With `distributed: true` every
  // node forms its own torch.distributed world (peer memory and NVLink stay inside a node): the
  // nodes' slot blocks must be aligned power-of-two blocks, this node's first, and the planner's
  // degrees are capped at the smallest block so that no group crosses a node
  std::vector<int> node_base(gpus, 0), node_size(gpus, gpus);
  std::vector<std::string> node_key(gpus);
  std::map<std::string, std::vector<int>> nodes;
  for (int g = 0; g < gpus; ++g) {
    node_key[g] = remote.count(g) ? remote_slots.at(std::to_string(g)).at("address").as_string() : std::string();
    nodes[node_key[g]].push_back(g);
  }
  if (distributed && nodes.size() > 1) {
    int smallest = gpus;
    for (const auto& [key, slots] : nodes) {
      const int b = slots.front(), k = static_cast<int>(slots.size());
      const bool contiguous = slots.back() - b + 1 == k;
      if (!contiguous || (k & (k - 1)) != 0 || b % k != 0)
        throw std::invalid_argument("with distributed: true each node's slots must form an aligned power-of-two block");
      if (key.empty() && b != 0) throw std::invalid_argument("this node's slots must come first");
      for (int g : slots) {
        node_base[g] = b;
        node_size[g] = k;
      }
      smallest = std::min(smallest, k);
    }
    if (transport != "collective" && transport != "export") throw std::invalid_argument("bad sp_transport");
    if (!options.contains("degrees")) {
      Json deg = Json::array();
      for (int d = 1; d <= smallest; d *= 2) deg.push_back(d);
      options["degrees"] = deg;
    }
  }
  auto lr = [&](int g) { return g - node_base[g]; };  // rank inside its node's world
  auto lranks = [&](const std::vector<int>& v) {
    Json a = Json::array();
    for (int g : v) a.push_back(lr(g));
    return a;
  };
  const std::string path = phase.str("collectives", "fused");
  const int batch_quantum = static_cast<int>(phase.integer("batch_quantum_steps", 4));
  // decode: finished videos run the VAE in chunked quanta (decode_start / decode_poll) and
  // images decode in finish; off: finish persists the final latents only
  const bool decode = phase.flag("decode", false);
  // decode_parallel: a finished video decodes on the group that ran its last step, patch
  // parallel (every member decodes its rows, halo rows over peer memory), in one quantum
  const bool decode_parallel = decode && phase.flag("decode_parallel", false);
  const size_t trace_limit = static_cast<size_t>(phase.integer("trace_limit", 2000));
  auto is_gpu = [](const Json& d) { return d.at("backend").as_string() != "mock"; };

  auto spawn = [&](const Json& def, const std::string& tag, int gidx, bool world_member) {
    Json d = def;
    const bool gpu = is_gpu(def);
    std::string visible = gpu ? std::to_string(gidx) : "";
    if (remote.count(gidx)) {
      const Json& rs = remote_slots.at(std::to_string(gidx));
      d["remote"] = rs.at("address");
      Json env = Json::object();
      if (gpu && world_member) {  // the node's world: every device of the node visible, ours by index
        std::string all;
        for (int h : nodes[node_key[gidx]])
          all += (all.empty() ? "" : ",") + remote_slots.at(std::to_string(h)).str("device", std::to_string(h));
        env["CUDA_VISIBLE_DEVICES"] = all;
        Json c = d.get("config").is_null() ? Json::object() : d.at("config");
        if (!c.contains("device")) c["device"] = "cuda:" + std::to_string(lr(gidx));
        d["config"] = c;
      } else {
        env["CUDA_VISIBLE_DEVICES"] = gpu ? rs.str("device", std::to_string(gidx)) : "";
      }
      d["remote_env"] = env;
      return spawn_worker(d, opt, run_dir + "/" + tag + std::to_string(gidx) + ".log", "");
    }
    Json c = d.get("config").is_null() ? Json::object() : d.at("config");
    if (world_member && gpu && !c.contains("device")) {  // peers' memory must be visible (IPC / NVLink)
      c["device"] = "cuda:" + std::to_string(gidx);
      d["config"] = c;
      visible = "all";
    }
    return spawn_worker(d, opt, run_dir + "/" + tag + std::to_string(gidx) + ".log", visible);
  };
  std::vector<std::unique_ptr<Worker>> vworkers, iworkers;
  for (int g = 0; g < gpus; ++g) {
    vworkers.push_back(spawn(vdef, "video", g, distributed));
    if (iname != vname) iworkers.push_back(spawn(idef, "image", g, false));
  }
  // occupancy guard: a CPU-only probe worker lists GPU processes that are not ours; a foreign
  // process on one of the phase's GPUs aborts the phase, and so do three unknown probes in a row
  const bool guard = phase.flag("occupancy_guard", false);
  const double guard_interval_ms = phase.num("occupancy_interval_ms", 5000.0);
  std::unique_ptr<WorkerProcess> prober;
  Json own_pids = Json::array();
  if (guard) {
    for (auto& w : vworkers) own_pids.push_back(static_cast<long long>(w->proc->pid()));
    for (auto& w : iworkers) own_pids.push_back(static_cast<long long>(w->proc->pid()));
    std::map<std::string, std::string> env;
    if (!opt.package_root.empty()) env["PYTHONPATH"] = opt.package_root;
    env["CUDA_VISIBLE_DEVICES"] = "";
    prober = std::make_unique<WorkerProcess>(
        std::vector<std::string>{opt.python, "-m", "ditserve_b200.runtime.worker", "--backend", "environment"}, env,
        run_dir + "/occupancy.log");
    prober->call("hello", Json::object(), 120);
  }
  auto W = [&](int g, bool image) -> Worker* {
    return (image && !iworkers.empty()) ? iworkers[g].get() : vworkers[g].get();
  };
  // ControllerTiming: one bounded span per worker call made for a quantum
  const size_t span_limit = static_cast<size_t>(phase.integer("span_limit", 4096));
  std::mutex span_mu;
  Json spans = Json::array();
  long long spans_dropped = 0;
  double t_origin = monotonic_seconds();
  auto call = [&](int g, bool image, const std::string& op, const Json& req) -> Json {
    const double a = monotonic_seconds();
    std::string status = "ok";
    Json res;
    try {
      res = W(g, image)->call(op, req);
    } catch (const std::exception& e) {
      status = std::string("error: ") + e.what();
    }
    const double b = monotonic_seconds();
    {
      std::lock_guard<std::mutex> lock(span_mu);
      if (spans.size() < span_limit) {
        Json sp = Json::object();
        sp["stage"] = op;
        sp["gpu"] = g;
        sp["worker"] = image ? "image" : "video";
        if (req.contains("state_id")) sp["request_id"] = req.at("state_id");
        sp["start_ms"] = (a - t_origin) * 1000.0;
        sp["finish_ms"] = (b - t_origin) * 1000.0;
        sp["status"] = status;
        if (res.is_object() && res.contains("model_ms")) sp["model_ms"] = res.at("model_ms");
        spans.push_back(sp);
      } else {
        ++spans_dropped;
      }
    }
    if (status != "ok") throw std::runtime_error(status.substr(7));
    return res;
  };
  if (distributed) {
    // one world per node, each rendezvousing on its own node's loopback
    std::map<std::string, int> node_port;
    int next_port = static_cast<int>(phase.integer("dist_port", 29700));
    for (const auto& kv : nodes) node_port[kv.first] = next_port++;
    std::vector<int> all;
    for (int g = 0; g < gpus; ++g) all.push_back(g);
    fan_out(all, [&](int g) {
      Json r = Json::object();
      r["action"] = "init";
      r["init_method"] = "tcp://127.0.0.1:" + std::to_string(node_port[node_key[g]]);
      r["rank"] = lr(g);
      r["world_size"] = node_size[g];
      r["timeout_s"] = phase.num("dist_timeout_s", 120.0);
      return vworkers[g]->call("distributed", r, 300);
    });
  }
  // untimed warm-up: every aligned group of each listed form adopts its layout once, so
  // communicators, symmetric heaps and fused plans exist before the trace starts
  double warmup_ms = 0;
  const double tw = monotonic_seconds();
  if (distributed && phase.contains("warmup_forms")) {
    Json spec = phase.get("warmup_spec").is_null() ? Json::object() : phase.at("warmup_spec");
    // "auto": every form the policy may choose for the phase's video classes
    std::vector<std::string> names;
    if (phase.at("warmup_forms").is_string() && phase.at("warmup_forms").as_string() == "auto") {
      std::set<std::string> seen;
      const Json gen = phase.get("generator");
      if (gen.is_object() && gen.contains("classes"))
        for (const auto& c : gen.at("classes").as_array()) {
          if (c.str("kind", "video") != "video") continue;
          for (const auto& f : candidate_forms(policy_traits(policy), cost, c.at("class").as_string(), gpus, options))
            if (f.degree() > 1 && seen.insert(form_name(f)).second) names.push_back(form_name(f));
        }
    } else {
      for (const auto& fj : phase.at("warmup_forms").as_array()) names.push_back(fj.as_string());
    }
    for (const auto& name : names) {
      const Form f = parse_form(name);
      for (const auto& grp : cluster_groups(gpus, f.degree())) {
        fan_out(grp, [&](int g) {
          Json r = Json::object();
          r["action"] = "layout";
          r["ranks"] = lranks(grp);
          r["form"] = form_name(f);
          r["spec"] = spec;
          r["path"] = path;
          return vworkers[g]->call("distributed", r, 600);
        });
      }
    }
  }
  // image workers: one short request each, so the first timed image pays no start-up
  if (phase.contains("warmup_image_spec") && !iworkers.empty()) {
    std::vector<int> all;
    for (int g = 0; g < gpus; ++g) all.push_back(g);
    fan_out(all, [&](int g) {
      Json pr = Json::object();
      pr["state_id"] = "__warmup__";
      pr["spec"] = phase.at("warmup_image_spec");
      iworkers[g]->call("prepare", pr, 600);
      Json ab = Json::object();
      Json ids = Json::array();
      ids.push_back("__warmup__");
      ab["state_ids"] = ids;
      iworkers[g]->call("advance_batch", ab, 600);  // warm-up specs take one step
      if (decode) {
        Json f = Json::object();
        f["state_id"] = "__warmup__";
        f["output_mode"] = "digest";
        f["decode"] = true;
        iworkers[g]->call("finish", f, 600);
      }
      Json rel = Json::object();
      rel["state_id"] = "__warmup__";
      return iworkers[g]->call("release", rel, 600);
    });
  }
  warmup_ms = (monotonic_seconds() - tw) * 1000.0;
  // doorbells: one 8-byte epoch file per GPU
  std::vector<std::string> bells;
  std::vector<long long> bell_epoch(gpus, 0);
  for (int g = 0; g < gpus; ++g) {
    bells.push_back(run_dir + "/doorbell" + std::to_string(g));
    std::ofstream(bells.back(), std::ios::binary).write("\0\0\0\0\0\0\0\0", 8);
  }
  auto ring = [&](int g) {
    ++bell_epoch[g];
    FILE* f = std::fopen(bells[g].c_str(), "r+b");
    if (!f) return;
    unsigned char b[8];
    unsigned long long v = static_cast<unsigned long long>(bell_epoch[g]);
    for (int i = 0; i < 8; ++i) b[i] = static_cast<unsigned char>((v >> (8 * i)) & 0xff);
    std::fwrite(b, 1, 8, f);
    std::fclose(f);
  };

  Json rows = study_workload(phase);
  std::vector<Live> live;
  std::map<std::string, size_t> idx;
  for (const auto& r : rows.as_array()) {
    Live l;
    l.row = r;
    l.id = r.at("request_id").as_string();
    l.kind = r.str("kind", "video");
    l.klass = r.str("class", l.kind);
    l.steps_total = static_cast<int>(r.at("spec").integer("steps", cost.steps(l.klass)));
    idx[l.id] = live.size();
    live.push_back(l);
  }
  struct Task {
    std::vector<std::string> ids;
    std::future<Json> fut;
    std::vector<int> group;
  };
  std::vector<Task> tasks;
  std::vector<bool> busy(gpus, false);
  std::vector<std::vector<std::pair<std::string, bool>>> pending_release(gpus);
  const double t0 = monotonic_seconds();
  t_origin = t0;
  long long plans = 0, quanta = 0, preemptions = 0, transfers = 0, pairs = 0, batches = 0, held_mid_step = 0;
  double plan_ms_total = 0, plan_ms_max = 0;
  size_t finished = 0;
  const double horizon = phase.num("horizon_ms", 1e12);
  Json failures = Json::array();
  Json trace = Json::array();

  // -- state placement (runs inside a task; members of `exec` are reserved for it) ----------
  struct Placement {
    std::string id;
    Json spec;
    bool image = false, prepared = false;
    std::vector<int> exec;
    std::set<int> fresh, stale;
  };
  auto ensure_state = [&, transport, path](const Placement& p) -> bool {
    if (!p.prepared) {
      fan_out(p.exec, [&](int g) {
        Json pr = Json::object();
        pr["state_id"] = p.id;
        pr["spec"] = p.spec;
        return call(g, p.image, "prepare", pr);
      });
      return false;
    }
    std::vector<int> need;
    for (int g : p.exec)
      if (!p.fresh.count(g)) need.push_back(g);
    if (need.empty()) return false;
    for (int g : need)
      if (p.stale.count(g)) {
        Json rel = Json::object();
        rel["state_id"] = p.id;
        call(g, p.image, "release", rel);
      }
    int src = -1;
    for (int g : p.exec)
      if (p.fresh.count(g)) {
        src = g;
        break;
      }
    auto hop = [&](int from, int to) {  // host-staged continuation packet
      Json ex = Json::object();
      ex["state_id"] = p.id;
      Json pk = call(from, p.image, "block_export", ex);
      Json im = pk;
      im["state_id"] = p.id;
      call(to, p.image, "block_import", im);
    };
    if (transport == "collective" && !p.image && p.exec.size() > 1) {
      if (src < 0) {
        hop(*p.fresh.begin(), p.exec.front());
        src = p.exec.front();
      }
      fan_out(p.exec, [&](int g) {
        Json r = Json::object();
        r["action"] = "migrate_group";
        r["ranks"] = lranks(p.exec);
        r["src"] = lr(src);
        r["state_id"] = p.id;
        r["path"] = path;
        return call(g, false, "distributed", r);
      });
    } else {
      const int from = src >= 0 ? src : *p.fresh.begin();
      for (int g : need) hop(from, g);
    }
    return true;
  };
  auto finish_release = [&](const std::string& id, const std::vector<int>& exec, bool image) {
    Json f = Json::object();
    f["state_id"] = id;
    f["output_mode"] = "digest";
    if (image && decode) f["decode"] = true;
    Json art = call(exec.front(), image, "finish", f);
    Json rel = Json::object();
    rel["state_id"] = id;
    fan_out(exec, [&](int g) { return call(g, image, "release", rel); });
    return art.get("value");
  };
  auto member = [](const std::string& id, const Json& progress, bool done, const Json& digest) {
    Json m = Json::object();
    m["id"] = id;
    m["progress"] = progress;
    m["finished"] = done;
    if (done) m["digest"] = digest;
    return m;
  };

  const size_t decision_plans = static_cast<size_t>(phase.integer("decision_plans", 64));
  Json decisions = Json::array();
  double next_probe = 0;
  int unknown_probes = 0;
  std::string abort_reason;
  Json probes = Json::array();
  // one occupancy verdict over the phase's GPUs: the local probe for this node's slots, and
  // each remote slot's bridge daemon for its GPU (the daemon excludes its own workers)
  auto probe_occupancy = [&]() -> Json {
    Json q = Json::object();
    Json probe_gpus = Json::array();
    for (int g = 0; g < gpus; ++g)
      if (!remote.count(g)) probe_gpus.push_back(g);
    q["gpus"] = probe_gpus;
    q["own_pids"] = own_pids;
    Json occ;
    try {
      occ = probe_gpus.empty() ? Json::object() : prober->call("occupancy", q, 60);
      if (probe_gpus.empty()) occ["state"] = "idle";
    } catch (const std::exception& e) {
      occ = Json::object();
      occ["state"] = "unknown";
      occ["source"] = e.what();
    }
    for (int g : remote) {
      const Json& rs = remote_slots.at(std::to_string(g));
      Json rq = Json::object();
      Json dev = Json::array();
      dev.push_back(std::stoi(rs.str("device", std::to_string(g))));
      rq["gpus"] = dev;
      std::string st = "unknown";
      Json r;
      try {
        r = vworkers[g]->call("bridge_occupancy", rq, 60);
        st = r.str("state", "unknown");
      } catch (const std::exception&) {
      }
      const std::string cur = occ.str("state", "unknown");
      if (st == "busy") {
        occ["state"] = "busy";
        if (!occ.contains("foreign") || !occ.at("foreign").is_object()) occ["foreign"] = Json::object();
        occ["foreign"]["remote-" + std::to_string(g)] = r.get("foreign");
      } else if (st == "unknown" && cur != "busy") {
        occ["state"] = "unknown";
      }
    }
    return occ;
  };
  // admission: with the guard on, the trace starts only once the phase's GPUs are idle
  double admission_wait_ms = 0;
  if (guard) {
    const double limit_s = phase.num("admission_wait_s", 60.0);
    const double ta = monotonic_seconds();
    std::string last_state = "unknown";
    while (true) {
      last_state = probe_occupancy().str("state", "unknown");
      if (last_state == "idle" || monotonic_seconds() - ta > limit_s) break;
      std::this_thread::sleep_for(std::chrono::milliseconds(500));
    }
    admission_wait_ms = (monotonic_seconds() - ta) * 1000.0;
    if (last_state != "idle") abort_reason = "admission: GPUs not idle (" + last_state + ")";
  }
  while (finished < live.size() && abort_reason.empty()) {
    const double now = now_ms_since(t0);
    if (now > horizon) break;
    if (guard && now >= next_probe) {
      next_probe = now + guard_interval_ms;
      const Json occ = probe_occupancy();
      const std::string st = occ.str("state", "unknown");
      if (probes.size() < 256) {
        Json pr = Json::object();
        pr["t_ms"] = now;
        pr["state"] = st;
        probes.push_back(pr);
      }
      unknown_probes = st == "unknown" ? unknown_probes + 1 : 0;
      if (st == "busy") abort_reason = "foreign GPU process: " + occ.get("foreign").dump();
      else if (unknown_probes > 2) abort_reason = "occupancy unknown on three probes in a row";
      if (!abort_reason.empty()) break;
    }
    // harvest finished quanta
    for (auto it = tasks.begin(); it != tasks.end();) {
      if (it->fut.wait_for(std::chrono::milliseconds(0)) != std::future_status::ready) {
        ++it;
        continue;
      }
      for (int g : it->group) busy[g] = false;
      Json res;
      std::string err;
      try {
        res = it->fut.get();
      } catch (const std::exception& e) {
        err = e.what();
      }
      for (const auto& id : it->ids) {
        Live& l = live[idx[id]];
        const Json* m = nullptr;
        if (err.empty())
          for (const auto& x : res.at("members").as_array())
            if (x.at("id").as_string() == id) m = &x;
        if (!err.empty() || m == nullptr) {
          l.status = "failed";
          l.row["status"] = "failed";
          l.row["error"] = err.empty() ? "no result for member" : err;
          failures.push_back(l.id);
          ++finished;
        } else {
          const Json& prog = m->get("progress");
          if (prog.is_object()) {
            l.steps_done = static_cast<int>(prog.integer("step", l.steps_done));
            l.blocks_done = static_cast<int>(prog.integer("block", 0));
            l.fold_eligible = prog.flag("cfg_fold_eligible", false);
          }
          if (m->contains("decode_ticket")) {
            l.decode_ticket = m->at("decode_ticket").as_string();
            l.decode_done = static_cast<int>(m->integer("decode_done", l.decode_done));
            l.decode_gpu = static_cast<int>(m->integer("decode_gpu", -1));
          }
          if (m->flag("finished", false)) {
            l.status = "done";
            l.row["status"] = "done";
            l.row["finish_ms"] = now_ms_since(t0);
            if (m->contains("digest")) l.row["digest"] = m->at("digest");
            ++finished;
          } else {
            l.status = "suspended";
          }
        }
        if (l.status == "done" || l.status == "failed") {
          for (int g : l.stale) pending_release[g].push_back({l.id, l.kind == "image"});
          if (l.status == "failed")
            for (int g : l.fresh) pending_release[g].push_back({l.id, l.kind == "image"});
          l.stale.clear();
          l.fresh.clear();
        }
        l.last_group = l.group;
        l.last_form = l.form;
        l.group.clear();
        l.rung = false;
      }
      it = tasks.erase(it);
    }
    // outdated copies on idle workers
    for (int g = 0; g < gpus; ++g) {
      if (busy[g] || pending_release[g].empty()) continue;
      for (const auto& pr : pending_release[g]) {
        Json rel = Json::object();
        rel["state_id"] = pr.first;
        try {
          W(g, pr.second)->call("release", rel, 60);
        } catch (const std::exception&) {
        }
      }
      pending_release[g].clear();
    }
    for (auto& l : live)
      if (l.status == "future" && l.row.at("arrival_ms").as_double() <= now) l.status = "waiting";
    // plan
    Json state = Json::object();
    state["now_ms"] = now;
    state["gpus"] = gpus;
    Json b = Json::array();
    for (bool x : busy) b.push_back(x);
    state["busy"] = b;
    Json reqs = Json::array();
    bool waiting = false;
    for (const auto& l : live) {
      if (l.status != "waiting" && l.status != "suspended" && l.status != "running") continue;
      waiting = waiting || l.status != "running";
      Json q = Json::object();
      q["request_id"] = l.id;
      q["kind"] = l.kind;
      q["class"] = l.klass;
      q["arrival_ms"] = l.row.at("arrival_ms");
      q["deadline_ms"] = l.row.at("deadline_ms");
      q["status"] = l.status;
      q["steps_total"] = l.steps_total;
      q["steps_done"] = l.steps_done;
      q["blocks_done"] = l.blocks_done;
      q["decode_done"] = l.decode_done;
      if (l.fold_eligible) q["cfg_fold_eligible"] = true;
      q["group"] = ints_json(l.status == "running" ? l.group : l.last_group);
      if (!l.form.empty()) q["form"] = l.form;
      // a started image keeps its GPU: its state lives in that GPU's image worker
      if (l.kind == "image" && l.status == "suspended" && !l.fresh.empty()) q["affinity"] = *l.fresh.begin();
      if (l.status == "running") {
        q["quantum_started_ms"] = l.quantum_started;
        q["rung"] = l.rung;
      }
      reqs.push_back(q);
    }
    state["requests"] = reqs;
    if (waiting) {
      const double tp = monotonic_seconds();
      // ControllerDecisions: the planner's ranking rows (laxity, feasibility) of the first
      // `decision_plans` plans; recording them cannot change a decision
      PlanTrace ptrace;
      const bool record = decisions.size() < decision_plans;
      Json plan = cluster_plan(state, policy, cost, options, record ? &ptrace : nullptr);
      if (record) {
        Json dj = Json::object();
        dj["t_ms"] = now;
        dj["ranking"] = ptrace.rows;
        dj["dropped"] = static_cast<long long>(ptrace.dropped);
        dj["assignments"] = static_cast<long long>(plan.at("assignments").size());
        dj["preempt"] = plan.at("preempt");
        decisions.push_back(dj);
      }
      const double pms = (monotonic_seconds() - tp) * 1000.0;
      plan_ms_total += pms;
      plan_ms_max = std::max(plan_ms_max, pms);
      ++plans;
      for (const auto& pid : plan.at("preempt").as_array()) {
        Live& l = live[idx[pid.as_string()]];
        if (l.status == "running" && !l.rung) {
          for (int g : l.group) ring(g);
          l.rung = true;
          ++preemptions;
        }
      }
      std::map<std::string, Json> by_id;
      for (const auto& a : plan.at("assignments").as_array()) by_id[a.at("request_id").as_string()] = a;
      std::set<std::string> handled;
      for (const auto& a : plan.at("assignments").as_array()) {
        const std::string rid = a.at("request_id").as_string();
        if (handled.count(rid)) continue;
        handled.insert(rid);
        Live& l = live[idx[rid]];
        if (l.status != "waiting" && l.status != "suspended") continue;
        std::vector<int> grp;
        for (const auto& gi : a.at("group").as_array()) grp.push_back(static_cast<int>(gi.as_int()));
        std::string form = a.at("form").as_string();
        const bool image = l.kind == "image";
        // a request inside a solver step keeps its group and form until the step ends
        if (!image && l.blocks_done > 0 && !l.last_group.empty() && (grp != l.last_group || form != l.last_form)) {
          grp = l.last_group;
          form = l.last_form;
          ++held_mid_step;
        }
        // a chunked decode continues on the worker that holds it
        if (!image && !l.decode_ticket.empty() && l.decode_gpu >= 0 && grp != std::vector<int>{l.decode_gpu})
          grp = std::vector<int>{l.decode_gpu};
        // a patch-parallel decode takes the group of the video's last step
        if (!image && decode_parallel && l.decode_ticket.empty() && l.steps_done >= l.steps_total &&
            !l.last_group.empty() && distributed)
          grp = l.last_group;
        bool free = true;
        for (int g : grp) free = free && !busy[g];
        if (!free) continue;
        // members of this quantum: a lockstep partner, or a continuous image batch
        std::vector<Live*> members{&l};
        const Json quantum = a.at("quantum");
        const std::string qs = quantum.is_string() ? quantum.as_string() : "";
        if (a.contains("pair") && !image) {
          const std::string pid = a.at("pair").as_string();
          Live& o = live[idx[pid]];
          if ((o.status == "waiting" || o.status == "suspended") && o.blocks_done == 0 && l.blocks_done == 0) {
            members.push_back(&o);
            handled.insert(pid);
          }
        }
        if (a.contains("batch"))
          for (const auto& x : a.at("batch").as_array()) {
            const std::string mid = x.as_string();
            if (mid == rid) continue;
            Live& o = live[idx[mid]];
            if (o.status != "waiting" && o.status != "suspended") continue;
            members.push_back(&o);
            handled.insert(mid);
          }
        const int leader = grp.front();
        const std::vector<int> exec = (distributed && !image) ? grp : std::vector<int>{leader};
        std::vector<Placement> places;
        for (Live* m : members) {
          Placement p;
          p.id = m->id;
          p.spec = m->row.at("spec");
          p.image = image;
          p.prepared = m->prepared;
          p.exec = exec;
          p.fresh = m->fresh;
          p.stale = m->stale;
          places.push_back(p);
          bool moves = m->prepared;
          if (moves) {
            bool all = true;
            for (int g : exec) all = all && m->fresh.count(g);
            moves = !all;
          }
          if (moves) ++transfers;
          for (int g : m->fresh)
            if (std::find(exec.begin(), exec.end(), g) == exec.end()) m->stale.insert(g);
          for (int g : exec) m->stale.erase(g);
          m->fresh = std::set<int>(exec.begin(), exec.end());
          m->prepared = true;
          m->status = "running";
          m->group = grp;
          m->form = form;
          m->quantum_started = now;
          if (!m->row.contains("start_ms")) m->row["start_ms"] = now;
        }
        for (int g : grp) busy[g] = true;
        ++quanta;
        if (members.size() > 1) (image ? batches : pairs) += 1;
        if (trace.size() < trace_limit) {
          Json tr = Json::object();
          tr["t_ms"] = now;
          tr["request_id"] = rid;
          tr["group"] = ints_json(grp);
          tr["form"] = form;
          tr["quantum"] = quantum;
          if (members.size() > 1) {
            Json ms = Json::array();
            for (Live* m : members) ms.push_back(m->id);
            tr["members"] = ms;
          }
          trace.push_back(tr);
        }
        std::vector<long long> epochs;
        for (int g = 0; g < gpus; ++g) epochs.push_back(bell_epoch[g]);
        std::vector<std::string> ids;
        for (Live* m : members) ids.push_back(m->id);
        const int degree = static_cast<int>(grp.size());
        const bool batch = a.contains("batch") || qs == "continuous_batch";
        const std::string ticket = l.decode_ticket;
        const int decoded = l.decode_done;
        const int chunks = std::max(1, cost.decode_chunks(l.klass));
        const int chunk_quantum = static_cast<int>(a.integer("decode_frames", chunks - decoded));
        const Json lspec = l.row.at("spec");
        const int frames = static_cast<int>(lspec.integer("frames", 81));
        const int latent_frames = (frames - 1) / 4 + 1;
        const int frames_per_chunk = (latent_frames + chunks - 1) / chunks;
        tasks.push_back({ids, std::async(std::launch::async, [=, &ensure_state, &finish_release, &member, &call,
                                                               &bells]() -> Json {
                           for (const auto& p : places) ensure_state(p);
                           Json out = Json::object();
                           Json ms = Json::array();
                           if (image) {
                             if (batch) {
                               Json ab = Json::object();
                               Json sids = Json::array();
                               for (const auto& id : ids) sids.push_back(id);
                               ab["state_ids"] = sids;
                               std::map<std::string, Json> prog;
                               for (int k = 0; k < batch_quantum; ++k) {
                                 Json r = call(leader, true, "advance_batch", ab);
                                 bool any = false;
                                 for (const auto& m : r.at("members").as_array()) {
                                   prog[m.at("state_id").as_string()] = m.at("progress");
                                   any = any || m.at("progress").flag("done", false);
                                 }
                                 if (any) break;
                               }
                               for (const auto& id : ids) {
                                 const bool done = prog[id].is_object() && prog[id].flag("done", false);
                                 ms.push_back(member(id, prog[id], done, done ? finish_release(id, exec, true) : Json()));
                               }
                             } else {
                               if (qs != "finish") {
                                 Json adv = Json::object();
                                 adv["state_id"] = ids[0];
                                 adv["steps"] = 1000000;
                                 call(leader, true, "advance", adv);
                               }
                               ms.push_back(member(ids[0], Json(), true, finish_release(ids[0], exec, true)));
                             }
                             out["members"] = ms;
                             return out;
                           }
                           if (qs == "finish") {
                             if (!decode) {
                               ms.push_back(member(ids[0], Json(), true, finish_release(ids[0], exec, false)));
                               out["members"] = ms;
                               return out;
                             }
                             if (decode_parallel && distributed && exec.size() > 1) {
                               // every member decodes its rows; the video is gathered on each
                               std::vector<Json> rs = fan_out(exec, [&](int g) {
                                 Json ds = Json::object();
                                 ds["state_id"] = ids[0];
                                 ds["group"] = lranks(grp);
                                 const std::string t = call(g, false, "decode_start", ds).at("ticket").as_string();
                                 Json dp = Json::object();
                                 dp["ticket"] = t;
                                 dp["wait"] = true;
                                 dp["output_mode"] = "digest";
                                 return call(g, false, "decode_poll", dp);
                               });
                               Json rel = Json::object();
                               rel["state_id"] = ids[0];
                               fan_out(exec, [&](int g) { return call(g, false, "release", rel); });
                               const Json& art = rs[0].get("artifact");
                               Json digest = art.is_object() && art.contains("array_sha256") ? art.at("array_sha256")
                                                                                            : rs[0].get("value");
                               ms.push_back(member(ids[0], Json(), true, digest));
                               out["members"] = ms;
                               return out;
                             }
                             std::string tk = ticket;
                             if (tk.empty()) {
                               Json ds = Json::object();
                               ds["state_id"] = ids[0];
                               ds["chunked"] = true;
                               tk = call(leader, false, "decode_start", ds).at("ticket").as_string();
                             }
                             Json dp = Json::object();
                             dp["ticket"] = tk;
                             dp["frames"] = std::max(1, chunk_quantum) * frames_per_chunk;
                             dp["output_mode"] = "digest";
                             if (decoded + chunk_quantum >= chunks) dp["wait"] = true;
                             Json r = call(leader, false, "decode_poll", dp);
                             if (r.flag("ready", false)) {
                               Json rel = Json::object();
                               rel["state_id"] = ids[0];
                               fan_out(exec, [&](int g) { return call(g, false, "release", rel); });
                               const Json& art = r.get("artifact");
                               Json digest = art.is_object() && art.contains("array_sha256") ? art.at("array_sha256")
                                                                                            : r.get("value");
                               Json m = member(ids[0], Json(), true, digest);
                               ms.push_back(m);
                             } else {
                               Json m = member(ids[0], Json(), false, Json());
                               m["decode_ticket"] = tk;
                               m["decode_done"] = std::min(chunks - 1, decoded + std::max(1, chunk_quantum));
                               m["decode_gpu"] = leader;
                               ms.push_back(m);
                             }
                             out["members"] = ms;
                             return out;
                           }
                           std::vector<Json> res = fan_out(exec, [&](int g) {
                             Json adv = Json::object();
                             adv["state_id"] = ids[0];
                             if (ids.size() > 1) adv["pair_state_id"] = ids[1];
                             adv["sp_degree"] = degree;
                             adv["group"] = ints_json(grp);
                             if (qs == "step") adv["quantum"] = "step";
                             else if (quantum.is_number()) adv["blocks"] = quantum;
                             else adv["quantum"] = "step";
                             Json bell = Json::object();
                             bell["path"] = bells[g];
                             bell["epoch"] = epochs[g];
                             adv["doorbell"] = bell;
                             if (distributed) {
                               Json lay = Json::object();
                               lay["ranks"] = lranks(grp);
                               lay["form"] = form;
                               lay["path"] = path;
                               adv["layout"] = lay;
                             }
                             return call(g, false, "advance", adv);
                           });
                           for (size_t k = 1; k < res.size(); ++k) {
                             const Json& p0 = res[0].at("progress");
                             const Json& pk = res[k].at("progress");
                             if (p0.integer("step", -1) != pk.integer("step", -1) ||
                                 p0.integer("block", 0) != pk.integer("block", 0))
                               throw std::runtime_error("SP group members diverged in progress");
                           }
                           for (size_t k = 0; k < ids.size(); ++k) {
                             const Json& prog = k == 0 ? res[0].at("progress") : res[0].at("pair_progress");
                             // with decode on, a denoised video waits for its own (chunked) decode quanta
                             const bool done = prog.flag("done", false) && !decode;
                             ms.push_back(member(ids[k], prog, done, done ? finish_release(ids[k], exec, false) : Json()));
                           }
                           out["members"] = ms;
                           return out;
                         }),
                         grp});
      }
    }
    std::this_thread::sleep_for(std::chrono::milliseconds(2));
  }
  for (auto& t : tasks) t.fut.wait();
  if (!abort_reason.empty())
    for (auto& l : live)
      if (l.status != "done" && l.status != "failed") {
        l.status = "failed";
        l.row["status"] = "failed";
        l.row["error"] = "aborted: " + abort_reason;
        failures.push_back(l.id);
      }
  if (prober) {
    try {
      prober->call("shutdown", Json::object(), 30);
    } catch (const std::exception&) {
    }
    prober->stop(2.0);
  }
  Json out_rows = Json::array();
  for (auto& l : live) {
    l.row["observation_ms"] = now_ms_since(t0);
    out_rows.push_back(l.row);
  }
  bool clean = true;
  auto stop_all = [&](std::vector<std::unique_ptr<Worker>>& ws) {
    for (auto& w : ws) {
      try {
        w->proc->call("shutdown", Json::object(), 30);
      } catch (const std::exception&) {
      }
      clean = w->proc->stop(5.0) && clean;
    }
  };
  stop_all(iworkers);
  stop_all(vworkers);
  Json out = Json::object();
  out["rows"] = out_rows;
  out["summary"] = request_summary(out_rows);
  Json c = Json::object();
  c["plans"] = plans;
  c["quanta"] = quanta;
  c["preemptions"] = preemptions;
  c["transfers"] = transfers;
  c["pairs"] = pairs;
  c["batches"] = batches;
  c["held_mid_step"] = held_mid_step;
  c["cleanup_verified"] = clean;
  out["counters"] = c;
  Json timing = Json::object();
  timing["plan_ms_total"] = plan_ms_total;
  timing["plan_ms_max"] = plan_ms_max;
  timing["wall_ms"] = now_ms_since(t0);
  timing["warmup_ms"] = warmup_ms;
  out["controller_timing"] = timing;
  out["trace"] = trace;
  out["spans"] = spans;
  if (guard) {
    out["occupancy_probes"] = probes;
    out["admission_wait_ms"] = admission_wait_ms;
    if (!abort_reason.empty()) out["aborted"] = abort_reason;
  }
  out["spans_dropped"] = spans_dropped;
  out["decisions"] = decisions;
  out["failures"] = failures;
  Json cfg = Json::object();
  cfg["distributed"] = distributed;
  cfg["sp_transport"] = transport;
  cfg["collectives"] = path;
  out["executor"] = cfg;
  return out;
}

Json run_simulate(const Json& phase) {
  const ClusterCost cost(phase.get("profile").is_null() ? synthetic_profile() : phase.at("profile"));
  std::unique_ptr<ClusterCost> pcost;
  if (phase.contains("planner_profile")) pcost = std::make_unique<ClusterCost>(phase.at("planner_profile"));
  const Json rows = study_workload(phase);
  const Json options = phase.get("options").is_null() ? Json::object() : phase.at("options");
  Json policies = phase.get("policies");
  if (policies.is_null()) {
    policies = Json::array();
    policies.push_back(phase.str("policy", "ditserve"));
  }
  Json out = Json::object();
  for (const auto& p : policies.as_array()) {
    SimResult r = simulate_cluster(rows, static_cast<int>(phase.integer("gpus", 8)), p.as_string(), cost, options,
                                   pcost.get());
    Json one = Json::object();
    one["summary"] = r.summary;
    one["counters"] = r.counters;
    if (phase.flag("keep_rows", false)) one["rows"] = r.rows;
    out[p.as_string()] = one;
  }
  return out;
}

}  // namespace

// ---------------------------------------------------------------------------------------
Json select_action(const Json& rows, double now_ms, const std::string& policy) {
  if (policy != "fcfs" && policy != "edf" && policy != "srtf") throw std::invalid_argument("policy must be fcfs, edf or srtf");
  Json d = select_online(rows, now_ms, policy);
  if (d.at("request_id").is_null()) throw std::invalid_argument("no request has arrived");
  d["policy"] = policy;
  return d;
}

Json synthetic_profile() {
  // B200 / NVSwitch default profile.  Video step times are measured SP1 steps of
  // this framework (both CFG branches, bench.py); images use SD3.5 estimates until
  // their calibration run replaces them (profiles/b200_profile.json).
  const char* text = R"JSON({
    "version": "ditserve-b200.profile.v1",
    "hardware": "8x B200, NVLink 5 / NVSwitch",
    "sp_efficiency": {"2": 0.97, "3": 0.95, "4": 0.94, "6": 0.9, "8": 0.88},
    "links": {"default_gbps": 700.0, "default_latency_ms": 0.02},
    "quantum_overhead_ms": 2.0, "block_overhead_ms": 0.05, "resize_ms": 5.0,
    "sp_overlap": 0.3, "pair_overlap": 0.2,
    "classes": {
      "wan21_480p": {"kind": "video", "steps": 50, "blocks_per_step": 30, "heads": 12,
                      "step_compute_ms": 686.0, "comm_mb_per_step": 24200.0, "collectives_per_step": 240,
                      "cfg_exchange_mb": 4.2, "decode_ms": 1500.0, "decode_chunks": 4},
      "wan22_720p": {"kind": "video", "steps": 50, "blocks_per_step": 30, "heads": 24,
                      "step_compute_ms": 1900.0, "comm_mb_per_step": 40200.0, "collectives_per_step": 240,
                      "ring_mb_per_step": 8000.0, "cfg_exchange_mb": 10.5, "decode_ms": 4000.0, "decode_chunks": 4},
      "sd35_512": {"kind": "image", "steps": 28, "tokens": 1024, "step_ms": 12.0, "service_ms": 420.0,
                   "decode_ms": 60.0, "batch_step_ms": {"1": 12.0, "2": 16.0, "4": 26.0, "8": 46.0}},
      "sd35_1024": {"kind": "image", "steps": 28, "tokens": 4096, "step_ms": 40.0, "service_ms": 1300.0,
                    "decode_ms": 180.0, "batch_step_ms": {"1": 40.0, "2": 74.0, "4": 142.0, "8": 280.0}}
    }})JSON";
  return Json::parse(text);
}

Json validate_study(const Json& config) {
  if (!config.is_object()) throw std::invalid_argument("study config must be an object");
  const std::string schema = config.str("schema", "");
  if (schema != "ditserve-b200.study.v1" && schema != "ditserve.study.v1")
    throw std::invalid_argument("study schema must be ditserve-b200.study.v1");
  const std::set<std::string> top = {"schema", "experiment", "workers", "budget", "phases", "description"};
  for (const auto& kv : config.as_object())
    if (!top.count(kv.first)) throw std::invalid_argument("unknown study key " + kv.first);
  if (!config.get("workers").is_object() || config.at("workers").empty())
    throw std::invalid_argument("study needs workers");
  for (const auto& kv : config.at("workers").as_object()) {
    const std::string b = kv.second.str("backend", "");
    if (b != "mock" && b != "wan" && b != "sd35") throw std::invalid_argument("worker " + kv.first + ": unknown backend");
  }
  std::set<std::string> ids;
  for (const auto& p : config.at("phases").as_array()) {
    const std::string id = p.at("id").as_string();
    if (id.empty() || id.find('/') != std::string::npos || !ids.insert(id).second)
      throw std::invalid_argument("phase ids must be unique safe path segments");
    const std::string kind = p.at("kind").as_string();
    if (kind != "operations" && kind != "online" && kind != "cluster" && kind != "simulate")
      throw std::invalid_argument("phase " + id + ": unknown kind " + kind);
    if (kind != "simulate") {
      std::vector<std::string> names;
      if (p.contains("workers")) {  // cluster phases: {"video": def, "image": def}
        if (kind != "cluster") throw std::invalid_argument("phase " + id + ": only cluster phases map workers by kind");
        for (const auto& kv : p.at("workers").as_object()) {
          if (kv.first != "video" && kv.first != "image")
            throw std::invalid_argument("phase " + id + ": workers keys are video and image");
          names.push_back(kv.second.as_string());
        }
      } else {
        names.push_back(p.str("worker", "model"));
      }
      for (const auto& n : names)
        if (!config.at("workers").contains(n)) throw std::invalid_argument("phase " + id + ": unknown worker " + n);
    }
    expand_matrix(p);  // validates axes and size
  }
  Json out = Json::object();
  out["valid"] = true;
  out["phases"] = static_cast<long long>(ids.size());
  out["identity"] = fnv1a(config.dump());
  return out;
}

Json run_study(const Json& config, const StudyOptions& opt) {
  const Json v = validate_study(config);
  const std::string identity = v.at("identity").as_string();
  const std::string run_id = opt.run_id.empty() ? config.str("experiment", "study") + "-" + identity : opt.run_id;
  const std::string dir = opt.work_dir + "/" + run_id;
  mkdirs(dir);
  const std::string run_json = dir + "/run.json";
  const Json code = code_identity(opt);
  if (exists(run_json)) {
    if (!opt.resume) throw std::runtime_error("run " + run_id + " exists; pass --resume to continue it");
    const Json prev = Json::parse(read_file(run_json));
    if (prev.at("identity").as_string() != identity)
      throw std::runtime_error("config changed since run " + run_id + " started; refusing to resume");
    if (prev.contains("code") && !(prev.at("code") == code))
      throw std::runtime_error("controller binary or worker sources changed since run " + run_id +
                               " started; refusing to resume");
  } else {
    Json r = Json::object();
    r["run_id"] = run_id;
    r["identity"] = identity;
    r["config"] = config;
    r["code"] = code;
    write_atomic(run_json, r.dump(1));
  }
  std::unique_ptr<Budget> budget;
  if (config.contains("budget")) {
    Json limits = Json::object();
    Json phases = Json::object();
    const Json& b = config.at("budget");
    for (const auto& p : config.at("phases").as_array()) {
      Json ph = Json::object();
      ph["gpu_seconds"] = b.get("phases").is_object() && b.at("phases").contains(p.at("id").as_string())
                              ? b.at("phases").at(p.at("id").as_string()).as_double()
                              : b.num("limit_gpu_seconds", 3600.0);
      phases[p.at("id").as_string()] = ph;
    }
    limits["phases"] = phases;
    limits["carry"] = b.str("carry", "none");
    limits["repair_reserve_gpu_seconds"] = b.num("repair_reserve_gpu_seconds", 0.0);
    budget = std::make_unique<Budget>(opt.ledger.empty() ? opt.work_dir + "/budget.json" : opt.ledger, limits);
  }
  Json report = Json::object();
  report["run_id"] = run_id;
  report["identity"] = identity;
  report["code"] = code;
  Json phases_out = Json::object();
  for (const auto& phase : config.at("phases").as_array()) {
    const std::string pid = phase.at("id").as_string();
    if (!opt.only_phase.empty() && pid != opt.only_phase) continue;
    const std::string result_path = dir + "/phase-" + pid + ".json";
    if (exists(result_path)) {
      phases_out[pid] = Json::parse(read_file(result_path));
      phases_out[pid]["resumed"] = true;
      continue;
    }
    const std::string kind = phase.at("kind").as_string();
    int devices = kind == "cluster" ? static_cast<int>(phase.integer("gpus", 8)) : 1;
    if (budget) budget->begin(identity + "/" + pid, devices, pid, config.at("budget").num("watchdog_seconds", 0), opt.repair);
    Json cells = expand_matrix(phase);
    std::vector<size_t> order;
    for (size_t i = 0; i < cells.size(); ++i) order.push_back(i);
    if (phase.flag("paired", false))
      for (size_t i = cells.size(); i-- > 0;) order.push_back(i);
    Json cell_results = Json::array();
    std::string status = "ok";
    bool cleanup = true;
    try {
      for (size_t k = 0; k < order.size(); ++k) {
        const Json& cell = cells[order[k]];
        Json res;
        if (kind == "simulate") {
          res = run_simulate(cell);
        } else if (kind == "cluster") {
          res = run_cluster(cell, opt, dir, config.at("workers"));
          cleanup = cleanup && res.at("counters").flag("cleanup_verified", true);
        } else {
          const Json& wdef = config.at("workers").at(cell.str("worker", "model"));
          auto w = spawn_worker(wdef, opt, dir + "/" + pid + "-cell" + std::to_string(k) + ".log", "");
          res = kind == "operations" ? run_operations(cell, *w) : run_online(cell, *w);
          try {
            w->proc->call("shutdown", Json::object(), 30);
          } catch (const std::exception&) {
          }
          cleanup = w->proc->stop(2.0) && cleanup;
        }
        if (budget) budget->check();
        Json cr = Json::object();
        cr["cell"] = cell.get("cell");
        cr["coordinates"] = cell.get("coordinates");
        cr["pass"] = static_cast<long long>(k < cells.size() ? 0 : 1);
        cr["result"] = res;
        cell_results.push_back(cr);
      }
    } catch (const std::exception& e) {
      status = std::string("failed: ") + e.what();
    }
    Json evidence = Json::object();
    evidence["cells"] = cell_results;
    evidence["status"] = status;
    if (cell_results.size() > 0) evidence["last"] = cell_results[cell_results.size() - 1].at("result");
    if (phase.contains("gates")) evidence["gates"] = evaluate_gates(evidence, phase.at("gates"));
    if (budget) evidence["budget"] = budget->finish(status == "ok" ? "ok" : "failed", cleanup);
    write_atomic(result_path, evidence.dump(1));
    phases_out[pid] = evidence;
    if (status != "ok") {
      report["phases"] = phases_out;
      report["status"] = status;
      return report;
    }
  }
  report["phases"] = phases_out;
  report["status"] = "ok";
  return report;
}

Json simulate_study(const Json& config) {
  Json out = Json::object();
  for (const auto& phase : config.at("phases").as_array()) {
    if (phase.at("kind").as_string() != "simulate" && phase.at("kind").as_string() != "cluster") continue;
    Json cells = expand_matrix(phase);
    Json res = Json::array();
    for (const auto& c : cells.as_array()) res.push_back(run_simulate(c));
    out[phase.at("id").as_string()] = res;
  }
  return out;
}

}  // namespace ds
