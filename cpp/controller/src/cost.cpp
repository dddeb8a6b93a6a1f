#include "ds/cost.hpp"

#include <algorithm>
#include <cmath>
#include <map>
#include <stdexcept>

namespace ds {

ClusterCost::ClusterCost(const Json& profile) : profile_(profile) {
  if (!profile_.is_object() || !profile_.get("classes").is_object())
    throw std::invalid_argument("cost profile needs a 'classes' object");
  resize_ms_ = profile_.num("resize_ms", 0.0);
  overhead_ms_ = profile_.num("quantum_overhead_ms", 0.0);
  block_overhead_ms_ = profile_.num("block_overhead_ms", 0.0);
  overlap_ = profile_.num("sp_overlap", 0.0);
  pair_overlap_ = profile_.num("pair_overlap", 0.0);
  for (const auto& kv : profile_.at("classes").as_object()) {
    const Json& c = kv.second;
    const std::string k = c.str("kind", "");
    if (k != "video" && k != "image") throw std::invalid_argument("class " + kv.first + ": kind must be video or image");
    if (k == "video" && !(c.num("step_compute_ms", -1) > 0) && !c.get("forms").is_object())
      throw std::invalid_argument("class " + kv.first + ": video needs step_compute_ms or measured forms");
    if (k == "image" && !(c.num("service_ms", -1) > 0))
      throw std::invalid_argument("class " + kv.first + ": image needs service_ms");
  }
  if (overlap_ < 0 || overlap_ > 1 || pair_overlap_ < 0 || pair_overlap_ > 1)
    throw std::invalid_argument("overlaps must lie in [0, 1]");
}

const Json& ClusterCost::klass(const std::string& name) const {
  const Json& c = profile_.at("classes").get(name);
  if (c.is_null()) throw std::invalid_argument("unknown request class: " + name);
  return c;
}
bool ClusterCost::has_class(const std::string& name) const { return profile_.at("classes").contains(name); }
std::string ClusterCost::kind(const std::string& name) const { return klass(name).at("kind").as_string(); }
int ClusterCost::steps(const std::string& name) const { return static_cast<int>(klass(name).integer("steps", 1)); }
int ClusterCost::blocks_per_step(const std::string& name) const {
  return static_cast<int>(klass(name).integer("blocks_per_step", 1));
}
int ClusterCost::heads(const std::string& name) const { return static_cast<int>(klass(name).integer("heads", 0)); }

double ClusterCost::efficiency(int sp) const {
  const Json& e = profile_.get("sp_efficiency");
  if (e.is_number()) return sp == 1 ? 1.0 : e.as_double();
  if (e.is_object()) {
    const Json& v = e.get(std::to_string(sp));
    if (!v.is_null()) return v.as_double();
  }
  return 1.0;
}

double ClusterCost::gbps(int sp, int sp_groups) const {
  const Json& l = profile_.get("links").get(std::to_string(sp));
  double rate = profile_.get("links").num("default_gbps", 700.0);
  if (l.is_object()) {
    rate = l.num("gbps", rate);
    const Json& cc = l.get("concurrent_gbps");
    if (cc.is_object() && sp_groups >= 2) {
      int best = 0;
      for (const auto& kv : cc.as_object()) {
        int k = std::stoi(kv.first);
        if (k <= sp_groups && k > best) {
          best = k;
          rate = kv.second.as_double();
        }
      }
    }
  }
  return rate;
}

double ClusterCost::latency_ms(int sp) const {
  const Json& l = profile_.get("links").get(std::to_string(sp));
  double lat = profile_.get("links").num("default_latency_ms", 0.01);
  if (l.is_object()) lat = l.num("latency_ms", lat);
  return lat;
}

ClusterCost::Terms ClusterCost::terms(const std::string& name, const Form& f, int sp_groups) const {
  const Json& c = klass(name);
  Terms t;
  const Json& measured = c.get("forms").get(form_name(f));
  if (measured.is_object() && measured.contains("step_ms")) {
    t.compute = measured.at("step_ms").as_double();
    t.measured = true;
    return t;
  }
  const double compute = c.num("step_compute_ms", 0.0);
  if (!(compute > 0)) throw std::invalid_argument("class " + name + " has no price for form " + form_name(f));
  const int sp = f.sp, cfg = f.cfg, ring = f.ring;
  t.compute = compute / (cfg * sp * efficiency(sp));
  if (sp > 1) {
    const double u = static_cast<double>(f.ulysses());
    t.comm = c.num("comm_mb_per_step", 0.0) / cfg * (u - 1.0) / (u * u) / gbps(sp, sp_groups) * (u / sp);
    t.latency = c.num("collectives_per_step", 0.0) / cfg * latency_ms(sp);
  }
  if (ring > 1) t.ring = c.num("ring_mb_per_step", 0.0) / cfg * (ring - 1.0) / (sp * ring) / gbps(ring, sp_groups);
  if (cfg == 2) t.exchange = c.num("cfg_exchange_mb", 0.0) / gbps(2, 1) + latency_ms(2);
  if (cfg == 1 && sp > 1) t.overlap = overlap_ * std::min(t.compute, t.comm);
  return t;
}

double ClusterCost::step_ms(const std::string& name, const Form& f, int sp_groups) const {
  return terms(name, f, sp_groups).total();
}

double ClusterCost::block_ms(const std::string& name, const Form& f, int sp_groups) const {
  const int blocks = blocks_per_step(name);
  return step_ms(name, f, sp_groups) / blocks + block_overhead_ms_ / f.cfg;
}

double ClusterCost::decode_ms(const std::string& name) const { return klass(name).num("decode_ms", 0.0); }
int ClusterCost::decode_chunks(const std::string& name) const {
  return std::max<int>(1, static_cast<int>(klass(name).integer("decode_chunks", 1)));
}

double ClusterCost::resume_ms(const std::string& name) const { return klass(name).num("resume_ms", 0.0); }

double ClusterCost::remaining_ms(const Json& r, const Form& f, int sp_groups) const {
  const std::string name = r.at("class").as_string();
  const int total = static_cast<int>(r.integer("steps_total", steps(name)));
  const int done = static_cast<int>(r.integer("steps_done", 0));
  const int blocks_done = static_cast<int>(r.integer("blocks_done", 0));
  if (kind(name) == "image") {
    const double per_step = image_step_ms(name);
    return std::max(0, total - done) * per_step + decode_ms(name) * (done >= total ? 0.0 : 0.0);
  }
  double ms = std::max(0, total - done) * step_ms(name, f, sp_groups);
  ms -= std::min(blocks_done, blocks_per_step(name)) * block_ms(name, f, sp_groups);
  const int decoded = static_cast<int>(r.integer("decode_done", 0));
  ms += std::max(0, decode_chunks(name) - decoded) * chunk_ms(name);
  return std::max(0.0, ms);
}

double ClusterCost::pair_ms(const std::string& a, const std::string& b, const Form& f) const {
  Terms ta = terms(a, f), tb = terms(b, f);
  const double sum = ta.total() + tb.total();
  const double hide = std::min(ta.compute + tb.compute, ta.comm + tb.comm + ta.latency + tb.latency);
  return sum - pair_overlap_ * hide;
}

double ClusterCost::service_ms(const std::string& name) const { return klass(name).at("service_ms").as_double(); }

double ClusterCost::image_step_ms(const std::string& name) const {
  const Json& c = klass(name);
  const double step = c.num("step_ms", 0.0);
  if (step > 0) return step;
  return (service_ms(name) - decode_ms(name)) / std::max(1, steps(name));
}

double ClusterCost::interp(const Json& table, double x) {
  std::map<double, double> pts;
  for (const auto& kv : table.as_object()) pts[std::stod(kv.first)] = kv.second.as_double();
  if (pts.empty()) throw std::invalid_argument("empty interpolation table");
  auto hi = pts.lower_bound(x);
  if (hi == pts.end()) {
    auto last = std::prev(pts.end());
    if (pts.size() == 1) return last->second * x / last->first;
    auto prev = std::prev(last);
    const double slope = (last->second - prev->second) / (last->first - prev->first);
    return last->second + slope * (x - last->first);
  }
  if (hi->first == x || hi == pts.begin()) return hi->second * (hi == pts.begin() && hi->first != x ? x / hi->first : 1.0);
  auto lo = std::prev(hi);
  const double w = (x - lo->first) / (hi->first - lo->first);
  return lo->second + w * (hi->second - lo->second);
}

double ClusterCost::batch_ms(const std::string& name, int size) const {
  const Json& t = klass(name).get("batch_ms");
  if (t.is_object()) return interp(t, size);
  return size * service_ms(name);
}

double ClusterCost::continuous_step_ms(const std::string& name, double eff) const {
  const Json& t = klass(name).get("batch_step_ms");
  if (t.is_object()) return interp(t, eff);
  return eff * image_step_ms(name);
}

double ClusterCost::effective_batch(const std::string& name, const std::vector<const Json*>& members,
                                    bool packing) const {
  // pixel-weighted size: a member counts tokens(member class) / tokens(batch class); without
  // packing every member is padded to the largest member of the batch
  const double base = std::max(1.0, klass(name).num("tokens", 1.0));
  double largest = 0, sum = 0;
  for (const Json* m : members) {
    const std::string c = m->str("class", name);
    const double tok = has_class(c) ? klass(c).num("tokens", base) : base;
    largest = std::max(largest, tok);
    sum += tok;
  }
  if (members.empty()) return 0.0;
  return packing ? sum / base : largest * members.size() / base;
}

std::string ClusterCost::batch_anchor(const std::vector<const Json*>& members, const std::string& fallback) const {
  std::string best = fallback;
  double best_tokens = -1;
  for (const Json* m : members) {
    const std::string c = m->str("class", fallback);
    const double tok = has_class(c) ? klass(c).num("tokens", 1.0) : 1.0;
    if (tok > best_tokens || (tok == best_tokens && c < best)) {
      best_tokens = tok;
      best = c;
    }
  }
  return best;
}

double ClusterCost::continuous_batch_step_ms(const std::vector<const Json*>& members, bool packing,
                                             const std::string& fallback) const {
  const std::string anchor = batch_anchor(members, fallback);
  return continuous_step_ms(anchor, effective_batch(anchor, members, packing));
}

}  // namespace ds
