// Cost model of one serving cluster: per-class, per-form step times.
//
// Analytical step time of a video class on form (cfg, sp, ring):
//   compute  = step_compute_ms / (cfg * sp * eff(sp))
//   comm     = comm_mb_per_step / cfg * (sp - 1) / sp^2 / gbps(sp)        (Ulysses all-to-all per rank)
//   ring     = ring_mb_per_step / cfg * (ring - 1) / (sp * ring) / gbps(ring)
//   latency  = [sp > 1] collectives_per_step / cfg * latency_ms(sp)
//   exchange = [cfg = 2] cfg_exchange_mb / gbps(2) + latency_ms(2)
//   step     = compute + comm + ring + latency + exchange - overlap * min(compute, comm)   (overlap: cfg = 1 only)
// MB / (GB/s) = ms.  A measured "forms": {name: {"step_ms": x}} entry of the class overrides
// the formula for that form.  On NVSwitch every rank subset sees the same link, so placement
// does not change the price; concurrent SP groups may still name a contention table
// (links.<sp>.concurrent_gbps {"k": gbps}).  Images: service_ms (atomic), batch_ms (atomic
// batches), batch_step_ms (continuous batching, one denoise round for k resident states,
// interpolated), tokens (for pixel-weighted packing).  Units: milliseconds.
// Same pricing structure as the reference (include/ditserve/control/cluster.hpp:33-54);
// our coefficients are calibrated on B200 (profiles/b200_profile.json).
#pragma once
#include <string>
#include <vector>

#include "ds/form.hpp"
#include "ds/json.hpp"

namespace ds {

class ClusterCost {
 public:
  explicit ClusterCost(const Json& profile);
  const Json& profile() const { return profile_; }
  const Json& klass(const std::string& name) const;
  bool has_class(const std::string& name) const;
  std::string kind(const std::string& name) const;  // video | image
  int steps(const std::string& name) const;
  int blocks_per_step(const std::string& name) const;
  int heads(const std::string& name) const;  // 0: unknown (no divisibility check)

  struct Terms {
    double compute = 0, comm = 0, ring = 0, latency = 0, exchange = 0, overlap = 0;
    bool measured = false;
    double total() const { return compute + comm + ring + latency + exchange - overlap; }
  };
  Terms terms(const std::string& klass, const Form& f, int sp_groups = 1) const;
  double step_ms(const std::string& klass, const Form& f, int sp_groups = 1) const;
  double block_ms(const std::string& klass, const Form& f, int sp_groups = 1) const;
  // remaining GPU-time on `f` from the request's progress (steps_done, blocks_done, decode_done)
  double remaining_ms(const Json& request, const Form& f, int sp_groups = 1) const;
  double decode_ms(const std::string& klass) const;
  int decode_chunks(const std::string& klass) const;
  double chunk_ms(const std::string& klass) const { return decode_ms(klass) / decode_chunks(klass); }
  // lockstep pair of two videos on one form: sum less pair_overlap of the shorter comm/compute
  double pair_ms(const std::string& a, const std::string& b, const Form& f) const;
  // images
  double service_ms(const std::string& klass) const;
  double batch_ms(const std::string& klass, int size) const;
  double continuous_step_ms(const std::string& klass, double effective_size) const;
  double effective_batch(const std::string& klass, const std::vector<const Json*>& members, bool packing) const;
  // the member class with the most tokens (ties: the smaller name); a mixed continuous batch is
  // priced on its table, so the price does not depend on which member anchors the batch
  std::string batch_anchor(const std::vector<const Json*>& members, const std::string& fallback) const;
  double continuous_batch_step_ms(const std::vector<const Json*>& members, bool packing,
                                  const std::string& fallback) const;
  double image_step_ms(const std::string& klass) const;
  double resume_ms(const std::string& klass) const;
  double resize_ms() const { return resize_ms_; }
  double overhead_ms() const { return overhead_ms_; }
  double block_overhead_ms() const { return block_overhead_ms_; }
  double pair_overlap() const { return pair_overlap_; }

 private:
  double efficiency(int sp) const;
  double gbps(int sp, int sp_groups) const;
  double latency_ms(int sp) const;
  static double interp(const Json& table, double x);
  Json profile_;
  double resize_ms_ = 0, overhead_ms_ = 0, block_overhead_ms_ = 0, overlap_ = 0, pair_overlap_ = 0;
};

}  // namespace ds
