#include "ds/rng.hpp"

#include <cmath>
#include <cstring>
#include <sstream>
#include <stdexcept>

namespace ds {

double Random::normal() {
  if (has_spare_) {
    has_spare_ = false;
    return spare_;
  }
  // Box-Muller: two independent normals from two uniforms
  const double u1 = uniform_open0();
  const double u2 = uniform();
  const double r = std::sqrt(-2.0 * std::log(u1));
  const double theta = 2.0 * M_PI * u2;
  spare_ = r * std::sin(theta);
  has_spare_ = true;
  return r * std::cos(theta);
}

double Random::exponential(double rate) {
  if (!(rate > 0.0)) throw std::invalid_argument("exponential rate must be positive");
  return -std::log(uniform_open0()) / rate;
}

double Random::gamma(double shape, double scale) {
  if (!(shape > 0.0) || !(scale > 0.0)) throw std::invalid_argument("gamma shape and scale must be positive");
  if (shape < 1.0) {
    // G(a) = G(a + 1) * U^(1/a)
    const double g = gamma(shape + 1.0, 1.0);
    return scale * g * std::pow(uniform_open0(), 1.0 / shape);
  }
  const double d = shape - 1.0 / 3.0;
  const double c = 1.0 / std::sqrt(9.0 * d);
  while (true) {
    double x, v;
    do {
      x = normal();
      v = 1.0 + c * x;
    } while (v <= 0.0);
    v = v * v * v;
    const double u = uniform_open0();
    if (u < 1.0 - 0.0331 * x * x * x * x) return scale * d * v;
    if (std::log(u) < 0.5 * x * x + d * (1.0 - v + std::log(v))) return scale * d * v;
  }
}

uint64_t Random::below(uint64_t n) {
  if (n == 0) throw std::invalid_argument("below(0)");
  // reject the 2^64 mod n smallest values so every residue is equally likely
  const uint64_t threshold = (0 - n) % n;
  uint64_t v;
  do {
    v = eng_();
  } while (v < threshold);
  return v % n;
}

Json Random::snapshot() const {
  std::ostringstream os;
  os << eng_;
  Json j = Json::object();
  j["version"] = kVersion;
  j["engine"] = os.str();
  j["has_spare"] = has_spare_;
  // the spare normal is stored bit-exactly as a hex integer string
  uint64_t bits;
  static_assert(sizeof bits == sizeof spare_, "double size");
  std::memcpy(&bits, &spare_, sizeof bits);
  j["spare_bits"] = std::to_string(bits);
  return j;
}

void Random::restore(const Json& snap) {
  if (snap.str("version", "") != kVersion) throw std::invalid_argument("RNG snapshot version mismatch");
  std::istringstream is(snap.at("engine").as_string());
  is >> eng_;
  if (is.fail()) throw std::invalid_argument("corrupt RNG engine state");
  has_spare_ = snap.at("has_spare").as_bool();
  uint64_t bits = std::stoull(snap.at("spare_bits").as_string());
  std::memcpy(&spare_, &bits, sizeof bits);
}

}  // namespace ds
