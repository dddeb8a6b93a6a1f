#include "ds/study.hpp"

#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <fstream>
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
#include "ds/planner.hpp"
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
  std::vector<std::string> argv = {def.str("python", opt.python), "-m", "ditserve_b200.runtime.worker",
                                   "--backend", backend, "--config",
                                   (def.get("config").is_null() ? Json::object() : def.at("config")).dump()};
  std::map<std::string, std::string> env;
  if (!opt.package_root.empty()) env["PYTHONPATH"] = opt.package_root;
  if (!gpu.empty()) env["CUDA_VISIBLE_DEVICES"] = gpu;
  else if (!gpu_backend) env["CUDA_VISIBLE_DEVICES"] = "";
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
  const int quantum = static_cast<int>(phase.integer("quantum_steps", 1));
  std::map<std::string, Json*> by_id;
  for (auto& r : rows.as_array()) by_id[r.at("request_id").as_string()] = &r;
  const double t0 = monotonic_seconds();
  std::set<std::string> prepared, done;
  std::map<std::string, double> remaining;
  while (done.size() < rows.size()) {
    const double now = now_ms_since(t0);
    Json visible = Json::array();
    double next_arrival = 1e300;
    for (const auto& r : rows.as_array()) {
      const std::string id = r.at("request_id").as_string();
      if (done.count(id)) continue;
      if (r.at("arrival_ms").as_double() > now) {
        next_arrival = std::min(next_arrival, r.at("arrival_ms").as_double());
        continue;
      }
      Json v = r;
      v["remaining_ms"] = remaining.count(id) ? remaining[id] : r.at("service_ms").as_double();
      visible.push_back(v);
    }
    if (visible.empty()) {
      std::this_thread::sleep_for(std::chrono::duration<double, std::milli>(std::max(0.0, next_arrival - now)));
      continue;
    }
    const std::string id = select_action(visible, now, policy).at("request_id").as_string();
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
    adv["steps"] = quantum;
    Json res = w.call("advance", adv);
    const Json& prog = res.at("progress");
    const double frac = prog.at("steps").as_double() > 0 ? prog.at("step").as_double() / prog.at("steps").as_double() : 1;
    remaining[id] = row.at("service_ms").as_double() * (1 - frac);
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
    }
  }
  for (auto& r : rows.as_array()) r["observation_ms"] = now_ms_since(t0);
  Json out = Json::object();
  out["rows"] = rows;
  out["summary"] = request_summary(rows);
  return out;
}

// ---------------------------------------------------------------------------------------
// multi-GPU executor: one worker per GPU slot; cluster_plan at every event
struct Live {
  std::string id, kind, klass, status = "future";
  Json row;
  int steps_total = 1, steps_done = 0, blocks_done = 0;
  std::vector<int> group, last_group;
  std::string form;
  int owner = -1;  // GPU whose worker holds the state
  bool prepared = false;
  double quantum_started = 0;
  bool rung = false;
};

Json run_cluster(const Json& phase, const StudyOptions& opt, const std::string& run_dir, const Json& workers_def) {
  const int gpus = static_cast<int>(phase.integer("gpus", 8));
  const std::string policy = phase.str("policy", "ditserve");
  const Json options = phase.get("options").is_null() ? Json::object() : phase.at("options");
  const ClusterCost cost(phase.get("profile").is_null() ? synthetic_profile() : phase.at("profile"));
  const Json& wdef = workers_def.at(phase.str("worker", "model"));
  const bool gpu_backend = wdef.at("backend").as_string() != "mock";
  std::vector<std::unique_ptr<Worker>> workers;
  for (int gidx = 0; gidx < gpus; ++gidx)
    workers.push_back(spawn_worker(wdef, opt, run_dir + "/worker" + std::to_string(gidx) + ".log",
                                   gpu_backend ? std::to_string(gidx) : ""));
  // doorbells: one 8-byte epoch file per GPU
  std::vector<std::string> bells;
  std::vector<long long> bell_epoch(gpus, 0);
  for (int gidx = 0; gidx < gpus; ++gidx) {
    bells.push_back(run_dir + "/doorbell" + std::to_string(gidx));
    std::ofstream(bells.back(), std::ios::binary).write("\0\0\0\0\0\0\0\0", 8);
  }
  auto ring = [&](int gidx) {
    ++bell_epoch[gidx];
    FILE* f = std::fopen(bells[gidx].c_str(), "r+b");
    if (!f) return;
    unsigned char b[8];
    unsigned long long v = static_cast<unsigned long long>(bell_epoch[gidx]);
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
    std::string id;
    std::future<Json> fut;
    std::vector<int> group;
  };
  std::vector<Task> tasks;
  std::vector<bool> busy(gpus, false);
  const double t0 = monotonic_seconds();
  long long plans = 0, quanta = 0, preemptions = 0, transfers = 0;
  size_t finished = 0;
  const double horizon = phase.num("horizon_ms", 1e12);
  Json failures = Json::array();
  while (finished < live.size()) {
    const double now = now_ms_since(t0);
    if (now > horizon) break;
    // harvest
    for (auto it = tasks.begin(); it != tasks.end();) {
      if (it->fut.wait_for(std::chrono::milliseconds(0)) != std::future_status::ready) {
        ++it;
        continue;
      }
      Live& l = live[idx[it->id]];
      for (int gi : it->group) busy[gi] = false;
      try {
        Json res = it->fut.get();
        const Json& prog = res.get("progress");
        if (prog.is_object()) {
          l.steps_done = static_cast<int>(prog.at("step").as_int());
          l.blocks_done = static_cast<int>(prog.integer("block", 0));
        }
        if (res.flag("finished", false)) {
          l.status = "done";
          l.row["status"] = "done";
          l.row["finish_ms"] = now_ms_since(t0);
          ++finished;
        } else {
          l.status = "suspended";
        }
      } catch (const std::exception& e) {
        l.status = "failed";
        l.row["status"] = "failed";
        l.row["error"] = e.what();
        failures.push_back(l.id);
        ++finished;
      }
      l.last_group = l.group;
      l.group.clear();
      l.rung = false;
      it = tasks.erase(it);
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
      Json grp = Json::array();
      for (int gi : (l.status == "running" ? l.group : l.last_group)) grp.push_back(gi);
      q["group"] = grp;
      if (!l.form.empty()) q["form"] = l.form;
      if (l.status == "running") {
        q["quantum_started_ms"] = l.quantum_started;
        q["rung"] = l.rung;
      }
      reqs.push_back(q);
    }
    state["requests"] = reqs;
    if (waiting) {
      Json plan = cluster_plan(state, policy, cost, options);
      ++plans;
      for (const auto& pid : plan.at("preempt").as_array()) {
        Live& l = live[idx[pid.as_string()]];
        if (l.status == "running" && !l.rung) {
          for (int gi : l.group) ring(gi);
          l.rung = true;
          ++preemptions;
        }
      }
      for (const auto& a : plan.at("assignments").as_array()) {
        Live& l = live[idx[a.at("request_id").as_string()]];
        if (l.status != "waiting" && l.status != "suspended") continue;
        std::vector<int> grp;
        for (const auto& gi : a.at("group").as_array()) grp.push_back(static_cast<int>(gi.as_int()));
        bool free = true;
        for (int gi : grp) free = free && !busy[gi];
        if (!free) continue;
        const int leader = grp.front();
        // exact state transfer when the request moves to another worker
        const bool move = l.prepared && l.owner >= 0 && l.owner != leader;
        const int from = l.owner;
        l.status = "running";
        l.group = grp;
        l.form = a.at("form").as_string();
        l.quantum_started = now;
        if (!l.row.contains("start_ms")) l.row["start_ms"] = now;
        for (int gi : grp) busy[gi] = true;
        if (move) ++transfers;
        const Json quantum = a.at("quantum");
        const Json spec = l.row.at("spec");
        const std::string id = l.id;
        const bool prepared = l.prepared;
        const long long epoch = bell_epoch[leader];
        const std::string bell = bells[leader];
        const int degree = static_cast<int>(grp.size());
        const bool image = l.kind == "image";
        Worker* dst = workers[leader].get();
        Worker* src = move ? workers[from].get() : nullptr;
        l.prepared = true;
        l.owner = leader;
        ++quanta;
        tasks.push_back({id, std::async(std::launch::async, [=]() -> Json {
                           if (src != nullptr) {
                             Json ex = Json::object();
                             ex["state_id"] = id;
                             Json pk = src->call("block_export", ex);
                             src->call("migration_release", ex);
                             Json im = Json::object();
                             im["state_id"] = id;
                             im["packet"] = pk.at("packet");
                             im["manifest"] = pk.at("manifest");
                             dst->call("block_import", im);
                           } else if (!prepared) {
                             Json pr = Json::object();
                             pr["state_id"] = id;
                             pr["spec"] = spec;
                             dst->call("prepare", pr);
                           }
                           Json adv = Json::object();
                           adv["state_id"] = id;
                           adv["sp_degree"] = degree;
                           if (quantum.is_string() && quantum.as_string() == "step") adv["quantum"] = "step";
                           else if (quantum.is_number()) adv["blocks"] = quantum;
                           else adv["steps"] = 1000000;  // atomic image / finish: run to the end
                           Json bellj = Json::object();
                           bellj["path"] = bell;
                           bellj["epoch"] = epoch;
                           adv["doorbell"] = bellj;
                           Json res;
                           const bool finish_only = quantum.is_string() && quantum.as_string() == "finish";
                           if (!finish_only) res = dst->call("advance", adv);
                           const bool done = finish_only || image || (res.get("progress").is_object() &&
                                                                     res.at("progress").flag("done", false));
                           if (done) {
                             Json f = Json::object();
                             f["state_id"] = id;
                             f["output_mode"] = "digest";
                             Json art = dst->call("finish", f);
                             dst->call("release", f);
                             Json out = Json::object();
                             out["finished"] = true;
                             out["digest"] = art.get("value");
                             return out;
                           }
                           return res;
                         }),
                         grp});
      }
    }
    std::this_thread::sleep_for(std::chrono::milliseconds(2));
  }
  for (auto& t : tasks) t.fut.wait();
  Json out_rows = Json::array();
  for (auto& l : live) {
    l.row["observation_ms"] = now_ms_since(t0);
    out_rows.push_back(l.row);
  }
  bool clean = true;
  for (auto& w : workers) {
    try {
      w->proc->call("shutdown", Json::object(), 30);
    } catch (const std::exception&) {
    }
    clean = w->proc->stop(2.0) && clean;
  }
  Json out = Json::object();
  out["rows"] = out_rows;
  out["summary"] = request_summary(out_rows);
  Json c = Json::object();
  c["plans"] = plans;
  c["quanta"] = quanta;
  c["preemptions"] = preemptions;
  c["transfers"] = transfers;
  c["cleanup_verified"] = clean;
  out["counters"] = c;
  out["failures"] = failures;
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
  if (!rows.is_array() || rows.empty()) throw std::invalid_argument("select_action needs visible requests");
  if (policy != "fcfs" && policy != "edf" && policy != "srtf") throw std::invalid_argument("online policy must be fcfs, edf or srtf");
  const Json* best = nullptr;
  auto key = [&](const Json& r) {
    const double arrival = r.num("arrival_ms", 0);
    double primary = arrival;
    if (policy == "edf") primary = r.num("deadline_ms", 1e300);
    if (policy == "srtf") primary = r.num("remaining_ms", 0);
    return std::make_tuple(primary, arrival, r.at("request_id").as_string());
  };
  for (const auto& r : rows.as_array()) {
    if (r.num("arrival_ms", 0) > now_ms) continue;
    if (best == nullptr || key(r) < key(*best)) best = &r;
  }
  if (best == nullptr) throw std::invalid_argument("no request has arrived");
  Json out = Json::object();
  out["request_id"] = best->at("request_id");
  out["policy"] = policy;
  return out;
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
    if (kind != "simulate" && !config.at("workers").contains(p.str("worker", "model")))
      throw std::invalid_argument("phase " + id + ": unknown worker");
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
  if (exists(run_json)) {
    if (!opt.resume) throw std::runtime_error("run " + run_id + " exists; pass --resume to continue it");
    const Json prev = Json::parse(read_file(run_json));
    if (prev.at("identity").as_string() != identity)
      throw std::runtime_error("config changed since run " + run_id + " started; refusing to resume");
  } else {
    Json r = Json::object();
    r["run_id"] = run_id;
    r["identity"] = identity;
    r["config"] = config;
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
