// Study runner: validated experiment configs executed phase by phase.
//
// config (schema "ditserve-b200.study.v1"; "ditserve.study.v1" accepted):
//   {experiment, workers: {name: {backend, config?, python?}}, budget: {phases|limit_gpu_seconds,
//    watchdog_seconds, repair_reserve_gpu_seconds, carry}, phases: [{id, kind, ...}]}
// phase kinds:
//   operations  a list of worker ops sent in order (optionally expecting failures)
//   online      one worker, requests replayed against the clock; select_online picks
//               which request advances next and for how many steps (benchmark orders,
//               session policies, EDF arms with fixed quanta, guarded / adaptive arms)
//   cluster     `gpus` workers (one per GPU), cluster_plan decides every quantum, calls
//               run concurrently, doorbells preempt block quanta, continuous batches
//   simulate    the discrete-event simulator over one or more policies
// A phase may carry a matrix (cartesian cells) and `paired: true` (cells run forward,
// then in reverse order, to cancel drift), and gates evaluated on its evidence.
// The run directory holds run.json (config hash + identity) and one result file per
// phase; --resume continues at the first phase without a result and refuses when the
// config changed.  Reference: src/ditserve/control/study.cpp:2257-2845.
#pragma once
#include <string>

#include "ds/json.hpp"

namespace ds {

struct StudyOptions {
  std::string run_id;
  std::string work_dir = "runs";
  std::string python = "python3";
  std::string package_root;  // PYTHONPATH for workers
  std::string ledger;        // budget ledger path (default <work_dir>/budget.json)
  std::string only_phase;
  bool resume = false;
  bool allow_gpu = false;
  bool repair = false;
};

Json validate_study(const Json& config);
Json run_study(const Json& config, const StudyOptions& opt);
Json simulate_study(const Json& config);
// online single-worker policy: which visible request acts next
// benchmark orders over rows {request_id, arrival_ms, deadline_ms, remaining_ms}
Json select_action(const Json& rows, double now_ms, const std::string& policy);
Json synthetic_profile();

}  // namespace ds
