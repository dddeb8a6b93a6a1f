// Workloads, serving metrics, gates and study matrices.
//
// study_workload(phase): a frozen request trace, either phase.workload rows or
// phase.generator = {count, seed, pattern offline_all|steady|poisson|bursty|gamma,
// rate_rps | rate_rpm, cv, burst_period_ms, burst_active_fraction, classes:[{weight,
// kind, class, spec, service_ms, slo_ms | slo_scale | slo_scale_range [lo, hi]}]}.
// Arrival and content streams use separate seeded generators so changing the
// class mixture never shifts arrival times.  Every row gets request_id,
// arrival_ms, service_ms, slo_ms, deadline_ms, kind, class, spec (with a seed).
//
// request_summary(rows): SLO attainment (on-time / all frozen requests, failed and
// unfinished included), goodput (on-time per second of exposure), latency
// p50/p95/p99 over finished requests, per-kind breakdowns.
// evaluate_gates(evidence, rules): [{pointer, op (<,<=,>,>=,==,!=), value}] on JSON pointers.
// expand_matrix(phase): cartesian product of phase.matrix.axes [{pointer, values}]
// applied to phase (at most 10 000 cells).
#pragma once
#include <string>

#include "ds/json.hpp"

namespace ds {

Json study_workload(const Json& phase);
Json request_summary(const Json& rows);
Json kind_summary(const Json& rows, const std::string& kind);
Json evaluate_gates(const Json& evidence, const Json& rules);
Json expand_matrix(const Json& phase);
double quantile(std::vector<double> v, double q);

// RFC 6901 JSON pointers
const Json* json_pointer_get(const Json& doc, const std::string& pointer);
void json_pointer_set(Json& doc, const std::string& pointer, const Json& value);

}  // namespace ds
