#include "ds/form.hpp"

#include <algorithm>
#include <cctype>
#include <stdexcept>

namespace ds {

namespace {
bool read_int(const std::string& s, size_t& i, int& out) {
  size_t j = i;
  while (j < s.size() && std::isdigit(static_cast<unsigned char>(s[j]))) ++j;
  if (j == i || j - i > 3) return false;
  out = std::stoi(s.substr(i, j - i));
  i = j;
  return out > 0;
}
}  // namespace

Form parse_form(const std::string& name) {
  Form f;
  size_t i = 0;
  if (name.compare(0, 4, "cfg2") == 0) {
    f.cfg = 2;
    i = 4;
  }
  if (i == name.size()) {
    if (f.cfg != 2) throw std::invalid_argument("bad form name: '" + name + "'");
    return f;
  }
  if (name.compare(i, 2, "sp") == 0) {
    i += 2;
    if (!read_int(name, i, f.sp)) throw std::invalid_argument("bad form name: '" + name + "'");
  } else if (name[i] == 'u') {
    ++i;
    int u = 0, r = 0;
    if (!read_int(name, i, u) || i >= name.size() || name[i] != 'r') throw std::invalid_argument("bad form name: '" + name + "'");
    ++i;
    if (!read_int(name, i, r)) throw std::invalid_argument("bad form name: '" + name + "'");
    f.sp = u * r;
    f.ring = r;
  } else {
    throw std::invalid_argument("bad form name: '" + name + "'");
  }
  if (i != name.size()) throw std::invalid_argument("bad form name: '" + name + "'");
  if (f.ring > 1 && f.sp < 4) throw std::invalid_argument("ring forms need sp >= 4: '" + name + "'");
  if (f.sp > 16) throw std::invalid_argument("sp degree too large: '" + name + "'");
  return f;
}

std::string form_name(const Form& f) {
  std::string base;
  if (f.ring > 1) base = "u" + std::to_string(f.ulysses()) + "r" + std::to_string(f.ring);
  else base = "sp" + std::to_string(f.sp);
  if (f.cfg == 2) return f.sp == 1 ? "cfg2" : "cfg2" + base;
  return base;
}

std::vector<Form> enumerate_forms(const std::vector<int>& sp_degrees, bool cfg_forms, bool ring_forms, int max_gpus) {
  std::vector<Form> out;
  for (int cfg : {1, 2}) {
    if (cfg == 2 && !cfg_forms) continue;
    for (int sp : sp_degrees) {
      for (int ring : {1, 2, 4}) {
        if (ring > 1 && (!ring_forms || sp < 4 || sp % ring != 0 || sp / ring < 1)) continue;
        Form f{cfg, sp, ring};
        if (f.degree() <= max_gpus) out.push_back(f);
      }
    }
  }
  std::sort(out.begin(), out.end());
  out.erase(std::unique(out.begin(), out.end()), out.end());
  return out;
}

}  // namespace ds
