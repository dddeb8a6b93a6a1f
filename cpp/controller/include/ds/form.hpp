// Parallel forms of one video request: CFG degree x sequence-parallel degree,
// the SP degree split into Ulysses x ring.  Names: sp1..sp8, cfg2, cfg2spK,
// uXrY, cfg2uXrY (the reference planner's vocabulary, kept so study configs
// and records stay interchangeable).  Here `sp` is the total sequence-parallel
// degree (ulysses * ring) and degree() = cfg * sp GPUs.
#pragma once
#include <string>
#include <vector>

namespace ds {

struct Form {
  int cfg = 1;
  int sp = 1;
  int ring = 1;
  int degree() const { return cfg * sp; }
  int ulysses() const { return sp / ring; }
  bool operator==(const Form& o) const { return cfg == o.cfg && sp == o.sp && ring == o.ring; }
  bool operator!=(const Form& o) const { return !(*this == o); }
  bool operator<(const Form& o) const {
    if (degree() != o.degree()) return degree() < o.degree();
    if (cfg != o.cfg) return cfg < o.cfg;
    return ring < o.ring;
  }
};

Form parse_form(const std::string& name);  // throws std::invalid_argument
std::string form_name(const Form& f);
// every form over the given SP degrees, optionally with cfg = 2 and ring forms
std::vector<Form> enumerate_forms(const std::vector<int>& sp_degrees, bool cfg_forms, bool ring_forms, int max_gpus);

}  // namespace ds
