// Command-line and RPC front end of the controller.
//
//   ditserve-b200 [--json] [--root P] [--python P] [--package-root P] COMMAND
//     doctor                                   environment facts (no CUDA init)
//     policies                                 the policy catalog
//     plan < state.json                        one cluster_plan decision
//     simulate [--config P] [--count N] [--seed N] [--policy ID]...
//     run --config P [--run-id ID] [--work-dir P] [--ledger P] [--phase ID] [--resume]
//     results finalize|verify|inspect|cleanup PATH | results compact ROOT DEST
//         [--allow-gpu] [--repair]
//     report RUN_DIR                           summaries of a finished run
//     rpc generate|simulate|control|plan|policies|run|simulate-study < request.json
// Exit codes: 0 success, 1 runtime failure, 2 usage error.
// `rpc generate|simulate|control|plan|policies` need no Python at all.
// Reference CLI: src/ditserve/interface/command.cpp:159-429.
#include <dirent.h>
#include <unistd.h>

#include <cstdlib>
#include <fstream>
#include <iostream>
#include <iterator>
#include <set>
#include <sstream>
#include <string>
#include <vector>

#include "ds/planner.hpp"
#include "ds/policy.hpp"
#include "ds/process.hpp"
#include "ds/sim.hpp"
#include "ds/cost.hpp"
#include "ds/dispatch.hpp"
#include "ds/study.hpp"
#include "ds/workload.hpp"

namespace ds {
namespace {

struct UsageError : std::invalid_argument {
  using std::invalid_argument::invalid_argument;
};

std::string slurp(std::istream& in, size_t cap) {
  std::string s;
  char buf[65536];
  while (in.read(buf, sizeof buf) || in.gcount() > 0) {
    s.append(buf, static_cast<size_t>(in.gcount()));
    if (s.size() > cap) throw UsageError("request exceeds 64 MiB");
  }
  return s;
}

std::string read_path(const std::string& p) {
  std::ifstream in(p);
  if (!in) throw std::runtime_error("cannot read " + p);
  return slurp(in, 64u << 20);
}

// phases may name a cost profile file ("profile_path", relative to the config file); it is
// inlined as "profile" so the study identity covers the profile's content
Json resolve_profiles(Json config, const std::string& config_path) {
  if (!config.contains("phases")) return config;
  std::string base = config_path;
  const size_t slash = base.find_last_of('/');
  base = slash == std::string::npos ? "." : base.substr(0, slash);
  Json phases = Json::array();
  for (const auto& ph : config.at("phases").as_array()) {
    Json p = ph;
    if (p.contains("profile_path") && !p.contains("profile")) {
      const std::string pp = p.at("profile_path").as_string();
      p["profile"] = Json::parse(read_path(!pp.empty() && pp[0] == '/' ? pp : base + "/" + pp));
    }
    phases.push_back(p);
  }
  config["phases"] = phases;
  return config;
}

Json pure_rpc(const std::string& cmd, const Json& req) {
  if (cmd == "policies") return policy_catalog();
  if (cmd == "generate") return study_workload(req);
  if (cmd == "plan") {
    const ClusterCost cost(req.get("profile").is_null() ? synthetic_profile() : req.at("profile"));
    return cluster_plan(req.at("state"), req.str("policy", "ditserve"), cost,
                        req.get("options").is_null() ? Json::object() : req.at("options"));
  }
  if (cmd == "control") {
    const std::string op = req.at("op").as_string();
    if (op == "select")
      return select_online(req.at("rows"), req.at("now_ms").as_double(), req.str("policy", "edf"),
                           req.str("active", ""), req.contains("quantum") ? req.at("quantum") : Json(1),
                           req.get("costs").is_null() ? Json::object() : req.at("costs"));
    if (op == "price") {  // the cost model's price of each named form of one class
      const ClusterCost cost(req.get("profile").is_null() ? synthetic_profile() : req.at("profile"));
      const std::string klass = req.at("class").as_string();
      Json out = Json::object();
      for (const auto& f : req.at("forms").as_array()) {
        const auto t = cost.terms(klass, parse_form(f.as_string()));
        Json row = Json::object();
        row["step_ms"] = t.total();
        row["measured"] = t.measured;
        row["compute"] = t.compute;
        row["comm"] = t.comm;
        row["latency"] = t.latency;
        row["exchange"] = t.exchange;
        row["overlap"] = t.overlap;
        out[f.as_string()] = row;
      }
      return out;
    }
    if (op == "workload") return study_workload(req.at("phase"));
    if (op == "matrix") return expand_matrix(req.at("phase"));
    if (op == "summary") return request_summary(req.at("rows"));
    if (op == "gates") return evaluate_gates(req.at("evidence"), req.at("rules"));
    throw UsageError("unknown control op " + op);
  }
  if (cmd == "simulate") {
    Json phase = req;
    phase["kind"] = "simulate";
    if (!phase.contains("id")) phase["id"] = "simulate";
    Json cfg = Json::object();
    cfg["phases"] = Json::array();
    cfg["phases"].push_back(phase);
    return simulate_study(cfg).at("simulate")[0];
  }
  if (cmd == "simulate-study") return simulate_study(req);
  throw UsageError("unknown rpc command " + cmd);
}

int usage(std::ostream& os) {
  os << "ditserve-b200 — native controller of the B200 DiT serving framework\n"
        "usage: ditserve-b200 [--json] [--root P] [--python P] [--package-root P] COMMAND\n"
        "  doctor | policies | plan < state.json\n"
        "  simulate [--config P] [--count N] [--seed N] [--policy ID]...\n"
        "  run --config P [--run-id ID] [--work-dir P] [--ledger P] [--phase ID] [--resume] [--allow-gpu] [--repair]\n"
        "  report RUN_DIR\n"
        "  results finalize RUN_DIR [--output DEST] [--title T] [--v1] | results verify|inspect PATH\n"
        "  results cleanup RUN_DIR --whitelist GLOB [...] [--dry-run] | results compact ROOT DEST [--prune-raw]\n"
        "  rpc generate|simulate|control|plan|policies|run|simulate-study < request.json\n";
  return 2;
}

}  // namespace

int command_main(int argc, char** argv) {
  std::vector<std::string> args(argv + 1, argv + argc);
  bool as_json = false;
  StudyOptions opt;
  if (const char* p = std::getenv("DITSERVE_PYTHON")) opt.python = p;
  if (const char* r = std::getenv("DITSERVE_PACKAGE_ROOT")) opt.package_root = r;
  std::vector<std::string> rest;
  try {
    for (size_t i = 0; i < args.size(); ++i) {
      const std::string& a = args[i];
      auto value = [&](const std::string& flag) -> std::string {
        const auto eq = a.find('=');
        if (eq != std::string::npos) return a.substr(eq + 1);
        if (i + 1 >= args.size()) throw UsageError("missing value for " + flag);
        return args[++i];
      };
      if (a == "--json") as_json = true;
      else if (a == "-h" || a == "--help") return usage(std::cout) - 2;
      else if (a.rfind("--python", 0) == 0) opt.python = value("--python");
      else if (a.rfind("--package-root", 0) == 0) opt.package_root = value("--package-root");
      else if (a.rfind("--root", 0) == 0) opt.work_dir = value("--root");
      else rest.push_back(a);
    }
    if (rest.empty()) return usage(std::cerr);
    const std::string cmd = rest[0];
    Json out;
    if (cmd == "rpc") {
      if (rest.size() != 2) throw UsageError("usage: ditserve-b200 rpc COMMAND < request.json");
      const std::string text = slurp(std::cin, 64u << 20);
      const Json req = Json::parse(text.empty() ? "{}" : text);
      if (rest[1] == "run") {
        StudyOptions o = opt;
        o.run_id = req.str("run_id", "");
        o.work_dir = req.str("work_dir", o.work_dir);
        o.resume = req.flag("resume", false);
        o.allow_gpu = req.flag("allow_gpu", false);
        out = run_study(req.at("config"), o);
      } else {
        out = pure_rpc(rest[1], req);
      }
      std::cout << out.dump() << "\n";
      return 0;
    }
    if (cmd == "policies") {
      out = policy_catalog();
    } else if (cmd == "plan") {
      out = pure_rpc("plan", Json::parse(slurp(std::cin, 64u << 20)));
    } else if (cmd == "doctor") {
      out = Json::object();
      out["controller"] = "ditserve-b200";
      out["policies"] = static_cast<long long>(policy_catalog().size());
      char host[256] = {0};
      gethostname(host, sizeof host - 1);
      out["host"] = host;
      out["python"] = opt.python;
      try {
        std::map<std::string, std::string> env;
        if (!opt.package_root.empty()) env["PYTHONPATH"] = opt.package_root;
        WorkerProcess w({opt.python, "-m", "ditserve_b200.runtime.worker", "--backend", "environment"}, env, "");
        out["worker"] = w.call("doctor", Json::object(), 120);
        w.call("shutdown", Json::object(), 30);
        w.stop(2.0);
      } catch (const std::exception& e) {
        out["worker_error"] = e.what();
      }
    } else if (cmd == "simulate") {
      Json phase = Json::object();
      std::vector<std::string> policies;
      for (size_t i = 1; i < rest.size(); ++i) {
        const std::string& a = rest[i];
        auto val = [&]() -> std::string {
          if (i + 1 >= rest.size()) throw UsageError("missing value for " + a);
          return rest[++i];
        };
        if (a == "--config") phase = Json::parse(read_path(val()));
        else if (a == "--count") phase["generator"]["count"] = std::stoll(val());
        else if (a == "--seed") phase["generator"]["seed"] = std::stoll(val());
        else if (a == "--policy") policies.push_back(val());
        else throw UsageError("unknown simulate option " + a);
      }
      if (!policies.empty()) {
        Json p = Json::array();
        for (auto& s : policies) p.push_back(s);
        phase["policies"] = p;
      }
      out = pure_rpc("simulate", phase);
    } else if (cmd == "run") {
      std::string config;
      for (size_t i = 1; i < rest.size(); ++i) {
        const std::string& a = rest[i];
        auto val = [&]() -> std::string {
          if (i + 1 >= rest.size()) throw UsageError("missing value for " + a);
          return rest[++i];
        };
        if (a == "--config") config = val();
        else if (a == "--run-id") opt.run_id = val();
        else if (a == "--work-dir") opt.work_dir = val();
        else if (a == "--ledger") opt.ledger = val();
        else if (a == "--phase") opt.only_phase = val();
        else if (a == "--resume") opt.resume = true;
        else if (a == "--allow-gpu") opt.allow_gpu = true;
        else if (a == "--repair") opt.repair = true;
        else throw UsageError("unknown run option " + a);
      }
      if (config.empty()) throw UsageError("run requires --config");
      out = run_study(resolve_profiles(Json::parse(read_path(config)), config), opt);
    } else if (cmd == "results") {
      // results finalize|verify|inspect PATH [--title T]; results compact ROOT DEST [--prune-raw]
      if (rest.size() < 3) throw UsageError("results needs an operation and a path");
      const std::string op = rest[1];
      Json req = Json::object();
      req["path"] = rest[2];
      size_t i = 3;
      if (op == "compact") {
        if (rest.size() < 4) throw UsageError("results compact needs ROOT and DEST");
        req["destination"] = rest[3];
        i = 4;
      } else if (op != "finalize" && op != "verify" && op != "inspect" && op != "cleanup") {
        throw UsageError("results operation must be finalize, verify, inspect, compact or cleanup");
      }
      Json whitelist = Json::array();
      for (; i < rest.size(); ++i) {
        if (rest[i] == "--title" && i + 1 < rest.size()) req["title"] = rest[++i];
        else if (rest[i] == "--output" && i + 1 < rest.size()) req["destination"] = rest[++i];
        else if (rest[i] == "--v1") req["format"] = "v1";
        else if (rest[i] == "--prune-raw") req["prune_raw"] = true;
        else if (rest[i] == "--whitelist" && i + 1 < rest.size()) whitelist.push_back(rest[++i]);
        else if (rest[i] == "--dry-run") req["dry_run"] = true;
        else throw UsageError("unknown results option " + rest[i]);
      }
      if (op == "cleanup") {
        if (whitelist.as_array().empty()) throw UsageError("results cleanup needs at least one --whitelist GLOB");
        req["whitelist"] = whitelist;
      }
      std::map<std::string, std::string> env;
      if (!opt.package_root.empty()) env["PYTHONPATH"] = opt.package_root;
      env["CUDA_VISIBLE_DEVICES"] = "";
      WorkerProcess w({opt.python, "-m", "ditserve_b200.runtime.worker", "--backend", "results"}, env, "");
      try {
        out = w.call(op, req, 600);
      } catch (...) {
        w.stop(2.0);
        throw;
      }
      w.call("shutdown", Json::object(), 30);
      w.stop(2.0);
    } else if (cmd == "report") {
      if (rest.size() != 2) throw UsageError("report needs exactly one RUN_DIR");
      out = Json::object();
      DIR* d = opendir(rest[1].c_str());
      if (!d) throw std::runtime_error("cannot open " + rest[1]);
      while (dirent* e = readdir(d)) {
        const std::string n = e->d_name;
        if (n.rfind("phase-", 0) != 0 || n.size() < 11 || n.substr(n.size() - 5) != ".json") continue;
        const Json ph = Json::parse(read_path(rest[1] + "/" + n));
        Json brief = Json::object();
        brief["status"] = ph.get("status");
        if (ph.contains("gates")) brief["gates_pass"] = ph.at("gates").at("pass");
        if (ph.get("last").is_object() && ph.at("last").contains("summary")) brief["summary"] = ph.at("last").at("summary");
        out[n.substr(6, n.size() - 11)] = brief;
      }
      closedir(d);
    } else {
      throw UsageError("unknown command " + cmd);
    }
    std::cout << (as_json ? out.dump() : out.dump(1)) << "\n";
    if (out.is_object() && out.contains("status") && out.at("status").is_string()) {
      // a run reports "ok"; results operations report what they did (finalized, cleaned, dry-run)
      // or why they did nothing (protected, deferred): the latter exit 1
      const std::string st = out.at("status").as_string();
      if (st != "ok" && st != "finalized" && st != "cleaned" && st != "dry-run") return 1;
    }
    return 0;
  } catch (const UsageError& e) {
    std::cerr << "usage error: " << e.what() << "\n";
    return 2;
  } catch (const JsonError& e) {
    std::cerr << "error: " << e.what() << "\n";
    return 2;
  } catch (const std::invalid_argument& e) {
    std::cerr << "error: " << e.what() << "\n";
    return 2;
  } catch (const std::exception& e) {
    std::cerr << "error: " << e.what() << "\n";
    return 1;
  }
}

}  // namespace ds

int main(int argc, char** argv) {
  ds::become_subreaper();
  return ds::command_main(argc, argv);
}
