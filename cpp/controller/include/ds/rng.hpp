// Deterministic, checkpointable random numbers for workload generation.
//
// Engine: std::mt19937_64 (its text serialisation is the standard's, so a
// snapshot restores the exact stream).  Normals use the Box-Muller transform
// with the spare value cached (and captured in snapshots); exponentials use
// inversion; bounded integers use rejection so every value is equally likely.
// Version tag: "mt19937_64-box-muller.v1".
#pragma once
#include <cstdint>
#include <random>
#include <string>

#include "ds/json.hpp"

namespace ds {

class Random {
 public:
  static constexpr const char* kVersion = "mt19937_64-box-muller.v1";
  explicit Random(uint64_t seed = 0) : eng_(seed) {}
  uint64_t next_u64() { return eng_(); }
  // uniform in [0, 1) with 53 random bits
  double uniform() { return static_cast<double>(eng_() >> 11) * (1.0 / 9007199254740992.0); }
  // uniform in (0, 1]
  double uniform_open0() { return 1.0 - uniform(); }
  double uniform(double lo, double hi) { return lo + (hi - lo) * uniform(); }
  double normal();
  double normal(double mean, double sd) { return mean + sd * normal(); }
  double exponential(double rate);
  // gamma(shape, scale) by Marsaglia & Tsang (2000), boosted for shape < 1
  double gamma(double shape, double scale);
  // unbiased integer in [0, n)
  uint64_t below(uint64_t n);

  Json snapshot() const;
  void restore(const Json& snap);

 private:
  std::mt19937_64 eng_;
  bool has_spare_ = false;
  double spare_ = 0.0;
};

}  // namespace ds
