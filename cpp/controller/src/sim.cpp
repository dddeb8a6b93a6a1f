#include "ds/sim.hpp"

#include <algorithm>
#include <cmath>
#include <limits>
#include <map>
#include <set>
#include <stdexcept>

#include "ds/planner.hpp"
#include "ds/workload.hpp"

namespace ds {
namespace {

struct SimReq {
  Json row;
  std::string id, kind, klass, status = "future";
  double arrival = 0, deadline = 0, finish = -1, start = -1;
  int steps_total = 1, steps_done = 0, blocks_done = 0, decode_done = 0;
  std::vector<int> group, last_group;
  std::string form;
  // running quantum
  double q_start = 0, q_end = 0;
  std::string q_kind;  // step | blocks | finish | atomic | batch
  int q_steps = 0, q_blocks = 0, q_decode = 0;
  std::vector<std::string> batch;  // continuous / atomic batch members (leader holds the list)
  std::string leader;              // member of someone else's batch
  bool rung = false;
  bool step_mode = false;  // image advanced step-wise (continuous batching)
};

}  // namespace

SimResult simulate_cluster(const Json& workload, int gpus, const std::string& policy, const ClusterCost& cost,
                           const Json& options, const ClusterCost* planner_cost, double horizon_ms) {
  const ClusterCost& pcost = planner_cost ? *planner_cost : cost;
  std::vector<SimReq> reqs;
  std::map<std::string, size_t> index;
  for (const auto& r : workload.as_array()) {
    SimReq s;
    s.row = r;
    s.id = r.at("request_id").as_string();
    s.kind = r.str("kind", "video");
    s.klass = r.str("class", s.kind);
    s.arrival = r.num("arrival_ms", 0.0);
    s.deadline = r.num("deadline_ms", 1e300);
    s.steps_total = static_cast<int>(r.integer("steps_total", cost.steps(s.klass)));
    index[s.id] = reqs.size();
    reqs.push_back(s);
  }
  std::vector<std::string> gpu_owner(gpus);
  long long plans = 0, quanta = 0, preemptions = 0, resizes = 0, batches = 0, batched_members = 0;
  double now = 0;
  const int max_events = 10000000;
  for (int ev = 0; ev < max_events; ++ev) {
    // next event time
    double next = std::numeric_limits<double>::infinity();
    for (const auto& r : reqs) {
      if (r.status == "future") next = std::min(next, r.arrival);
      if (r.status == "running" && r.leader.empty()) next = std::min(next, r.q_end);
    }
    if (!std::isfinite(next) || next > horizon_ms) break;
    now = std::max(now, next);
    // completions
    for (auto& r : reqs) {
      if (r.status != "running" || !r.leader.empty() || r.q_end > now) continue;
      auto finish_member = [&](SimReq& m, bool leader) {
        for (int gi : (leader ? m.group : std::vector<int>{})) gpu_owner[gi].clear();
        m.last_group = m.group.empty() ? m.last_group : m.group;
        if (m.q_kind == "step") {
          m.steps_done = std::min(m.steps_total, m.steps_done + m.q_steps);
          m.blocks_done = 0;
        } else if (m.q_kind == "blocks") {
          const int bps = cost.blocks_per_step(m.klass);
          m.blocks_done += m.q_blocks;
          while (m.blocks_done >= bps) {
            m.blocks_done -= bps;
            ++m.steps_done;
          }
        } else if (m.q_kind == "finish") {
          m.decode_done += m.q_decode;
        } else if (m.q_kind == "cstep") {
          ++m.steps_done;
        }
        bool done = false;
        if (m.kind == "image") {
          done = m.q_kind == "atomic" || m.q_kind == "finish" || (m.step_mode && m.steps_done >= m.steps_total);
        } else {
          done = m.steps_done >= m.steps_total && m.decode_done >= cost.decode_chunks(m.klass);
        }
        if (m.kind == "video" && m.steps_done >= m.steps_total && cost.decode_ms(m.klass) <= 0) done = true;
        m.status = done ? "done" : "suspended";
        if (done) m.finish = m.q_end;
        m.group.clear();
        m.rung = false;
        m.leader.clear();
      };
      for (const auto& mid : r.batch) {
        if (mid == r.id) continue;
        auto& m = reqs[index[mid]];
        m.q_end = r.q_end;
        m.q_kind = r.q_kind;
        finish_member(m, false);
      }
      finish_member(r, true);
      r.batch.clear();
    }
    // arrivals
    for (auto& r : reqs)
      if (r.status == "future" && r.arrival <= now) r.status = "waiting";
    // plan
    Json state = Json::object();
    state["now_ms"] = now;
    state["gpus"] = gpus;
    Json busy = Json::array();
    for (int i = 0; i < gpus; ++i) busy.push_back(!gpu_owner[i].empty());
    state["busy"] = busy;
    Json rj = Json::array();
    int sp_running = 0;
    for (const auto& r : reqs) {
      if (r.status != "waiting" && r.status != "suspended" && r.status != "running") continue;
      if (r.status == "running" && !r.leader.empty()) continue;
      Json q = Json::object();
      q["request_id"] = r.id;
      q["kind"] = r.kind;
      q["class"] = r.klass;
      q["arrival_ms"] = r.arrival;
      q["deadline_ms"] = r.deadline;
      q["status"] = r.status;
      q["steps_total"] = r.steps_total;
      if (r.kind == "video" || r.step_mode) q["steps_done"] = r.steps_done;
      q["blocks_done"] = r.blocks_done;
      q["decode_done"] = r.decode_done;
      Json grp = Json::array();
      for (int gi : (r.status == "running" ? r.group : r.last_group)) grp.push_back(gi);
      q["group"] = grp;
      if (!r.form.empty()) q["form"] = r.form;
      if (r.status == "running") {
        q["quantum_started_ms"] = r.q_start;
        q["rung"] = r.rung;
        if (r.group.size() > 1) ++sp_running;
      }
      rj.push_back(q);
    }
    state["requests"] = rj;
    state["sp_groups_running"] = sp_running;
    bool any_waiting = false;
    for (const auto& r : reqs) any_waiting = any_waiting || r.status == "waiting" || r.status == "suspended";
    if (!any_waiting) continue;
    Json plan = cluster_plan(state, policy, pcost, options);
    ++plans;
    // preemption: rung groups stop at their next doorbell check
    for (const auto& pid : plan.at("preempt").as_array()) {
      auto& r = reqs[index[pid.as_string()]];
      if (r.status != "running" || r.rung || r.kind != "video") continue;
      const Form f = parse_form(r.form);
      const double bms = cost.block_ms(r.klass, f);
      const double stop_at = now + bms * (f.sp > 1 ? 2 : 1);
      if (stop_at < r.q_end && (r.q_kind == "step" || r.q_kind == "blocks")) {
        const int executed = static_cast<int>(std::floor((stop_at - r.q_start) / bms));
        const int bps = cost.blocks_per_step(r.klass);
        const int total_blocks = r.blocks_done + std::min(executed, r.q_kind == "step" ? r.q_steps * bps : r.q_blocks);
        r.q_kind = "blocks";
        r.q_blocks = total_blocks - r.blocks_done;
        r.q_end = r.q_start + r.q_blocks * bms;
        if (r.q_end < now) r.q_end = now;
        ++preemptions;
      }
      r.rung = true;
    }
    for (const auto& a : plan.at("assignments").as_array()) {
      auto& r = reqs[index[a.at("request_id").as_string()]];
      if (r.status != "waiting" && r.status != "suspended") continue;
      std::vector<int> grp;
      for (const auto& gi : a.at("group").as_array()) grp.push_back(static_cast<int>(gi.as_int()));
      bool free = true;
      for (int gi : grp) free = free && gpu_owner[gi].empty();
      if (!free && !a.contains("pair")) continue;
      const Form f = parse_form(a.at("form").as_string());
      const bool resized = !r.last_group.empty() && r.last_group != grp;
      if (resized) ++resizes;
      double dur = cost.overhead_ms() + (resized ? cost.resize_ms() : 0.0);
      if (r.start < 0) r.start = now;
      const Json& qv = a.at("quantum");
      if (r.kind == "video") {
        if (!r.last_group.empty() && resized) dur += cost.resume_ms(r.klass);
        if (qv.is_string() && qv.as_string() == "finish") {
          const int chunks = cost.decode_chunks(r.klass);
          r.q_decode = static_cast<int>(a.integer("decode_frames", chunks - r.decode_done));
          r.q_kind = "finish";
          dur += r.q_decode * cost.chunk_ms(r.klass);
        } else if (qv.is_string()) {
          r.q_kind = "step";
          r.q_steps = static_cast<int>(a.integer("steps", 1));
          double step = cost.step_ms(r.klass, f);
          if (a.contains("pair")) {
            const auto& other = reqs[index[a.at("pair").as_string()]];
            step = cost.pair_ms(r.klass, other.klass, f) / 2.0;
          }
          dur += r.q_steps * step - r.blocks_done * cost.block_ms(r.klass, f);
        } else {
          r.q_kind = "blocks";
          r.q_blocks = static_cast<int>(qv.as_int());
          dur += r.q_blocks * cost.block_ms(r.klass, f);
        }
      } else {
        const std::string qk = qv.as_string();
        std::vector<std::string> members{r.id};
        if (a.contains("batch")) {
          members.clear();
          for (const auto& m : a.at("batch").as_array()) members.push_back(m.as_string());
        }
        if (qk == "continuous_batch") {
          std::vector<const Json*> js;
          for (const auto& m : members) js.push_back(&reqs[index[m]].row);
          const double round_ms =
              cost.continuous_batch_step_ms(js, options.flag("sequence_packing", true), r.klass);
          dur += round_ms;
          for (const auto& m : members) {
            auto& mm = reqs[index[m]];
            mm.step_mode = true;
            if (mm.steps_done + 1 >= mm.steps_total) dur = std::max(dur, round_ms + cost.decode_ms(mm.klass));
          }
          r.q_kind = "cstep";
        } else {
          r.q_kind = qk == "finish" ? "finish" : "atomic";
          dur += members.size() > 1 ? cost.batch_ms(r.klass, static_cast<int>(members.size())) : cost.service_ms(r.klass);
        }
        if (members.size() > 1) {
          ++batches;
          batched_members += static_cast<long long>(members.size());
        }
        r.batch = members;
        for (const auto& m : members) {
          if (m == r.id) continue;
          auto& mm = reqs[index[m]];
          if (mm.status != "waiting" && mm.status != "suspended") continue;
          mm.status = "running";
          mm.leader = r.id;
          mm.q_kind = r.q_kind;
          if (mm.start < 0) mm.start = now;
        }
      }
      r.status = "running";
      r.group = grp;
      r.form = a.at("form").as_string();
      r.q_start = now;
      r.q_end = now + std::max(0.0, dur);
      for (int gi : grp) gpu_owner[gi] = r.id;
      ++quanta;
    }
  }
  SimResult out;
  out.rows = Json::array();
  for (const auto& r : reqs) {
    Json row = r.row;
    row["status"] = r.status == "done" ? "done" : (r.status == "future" ? "not_executed" : "censored");
    if (r.finish >= 0) row["finish_ms"] = r.finish;
    if (r.start >= 0) row["start_ms"] = r.start;
    row["observation_ms"] = now;
    out.rows.push_back(row);
  }
  out.summary = request_summary(out.rows);
  out.counters = Json::object();
  out.counters["plans"] = plans;
  out.counters["quanta"] = quanta;
  out.counters["preemptions"] = preemptions;
  out.counters["resizes"] = resizes;
  out.counters["batches"] = batches;
  out.counters["batched_members"] = batched_members;
  out.counters["end_ms"] = now;
  return out;
}

}  // namespace ds
