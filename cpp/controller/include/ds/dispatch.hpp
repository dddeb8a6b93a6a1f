// Single-worker action selection for the online replay (one GPU, one request at a time).
//
// Policies:
//   fcfs | edf | srtf          benchmark orders (arrival, deadline, remaining work); the active
//                              request keeps the worker unless another one strictly precedes it
//                              (fcfs never switches away from the active request)
//   session_serial | stage_edf | session_slack
//                              session policies over ready rows: keep the active session,
//                              earliest stage deadline, or least slack (deadline - now - remaining)
//   edf_b1 | edf_b1_async | edf_b2 | edf_b4 | edf_step
//                              EDF with a fixed quantum (1, 2, 4 steps or a whole step)
//   guarded_b4 | guarded_adaptive | feasible_b4
//                              EDF over requests that can still meet their deadline, with
//                              (a) a waiting guard: a request ready for 2.5x its service time
//                                  is served first unless that endangers another deadline,
//                              (b) for guarded_*, a resume guard that lets a started video whose
//                                  slack would not survive the candidate's quantum go first,
//                              (c) a deadline-conflict fallback: EDF with the smallest quantum;
//                              guarded_adaptive picks the largest quantum in {1, 4, 8} (denoise
//                              only) whose cost fits the smallest slack of the others and half
//                              the image deadline (costs.image_deadline_ms)
// Row fields: request_id, kind, arrival_ms, deadline_ms, remaining_ms, service_ms, ready_since_ms,
// action (prepare|denoise|decode|image), started, action_ms_by_quantum {"1": ms, "4": ms, ...};
// session rows: release_ms, stage_deadline_ms, remaining_total_ms, ready.
// Decision: {request_id | null, quantum, reason, predicted_deadline_conflict, slack_ms}.
// Same decision rules as the reference's select_action (src/ditserve/control/dispatch.cpp:69-160).
#pragma once
#include <string>

#include "ds/json.hpp"

namespace ds {

Json select_online(const Json& rows, double now_ms, const std::string& policy, const std::string& active = "",
                   const Json& default_quantum = Json(1), const Json& costs = Json::object());

bool is_online_policy(const std::string& policy);

}  // namespace ds
