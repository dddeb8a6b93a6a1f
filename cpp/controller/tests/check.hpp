// Minimal test harness: named checks, failures counted, non-zero exit on failure.
#pragma once
#include <cmath>
#include <functional>
#include <iostream>
#include <string>
#include <vector>

namespace dstest {
struct Case {
  std::string name;
  std::function<void()> fn;
};
inline std::vector<Case>& cases() {
  static std::vector<Case> c;
  return c;
}
inline int& failures() {
  static int f = 0;
  return f;
}
struct Reg {
  Reg(const char* n, std::function<void()> f) { cases().push_back({n, f}); }
};
inline int run_all() {
  int failed_cases = 0;
  for (auto& c : cases()) {
    const int before = failures();
    try {
      c.fn();
    } catch (const std::exception& e) {
      std::cerr << "  exception in " << c.name << ": " << e.what() << "\n";
      ++failures();
    }
    const bool ok = failures() == before;
    failed_cases += !ok;
    std::cout << (ok ? "[ ok ] " : "[FAIL] ") << c.name << "\n";
  }
  std::cout << cases().size() - failed_cases << "/" << cases().size() << " checks passed\n";
  return failed_cases == 0 ? 0 : 1;
}
}  // namespace dstest

#define DS_CAT2(a, b) a##b
#define DS_CAT(a, b) DS_CAT2(a, b)
#define TEST(name) \
  static void DS_CAT(test_fn_, __LINE__)(); \
  static dstest::Reg DS_CAT(test_reg_, __LINE__)(name, DS_CAT(test_fn_, __LINE__)); \
  static void DS_CAT(test_fn_, __LINE__)()
#define CHECK(cond)                                                                              \
  do {                                                                                           \
    if (!(cond)) {                                                                               \
      std::cerr << "  " << __FILE__ << ":" << __LINE__ << ": CHECK failed: " #cond "\n";         \
      ++dstest::failures();                                                                      \
    }                                                                                            \
  } while (0)
#define CHECK_THROWS(expr)                                                                       \
  do {                                                                                           \
    bool thrown_ = false;                                                                        \
    try {                                                                                        \
      (void)(expr);                                                                              \
    } catch (...) {                                                                              \
      thrown_ = true;                                                                            \
    }                                                                                            \
    if (!thrown_) {                                                                              \
      std::cerr << "  " << __FILE__ << ":" << __LINE__ << ": expected exception: " #expr "\n";   \
      ++dstest::failures();                                                                      \
    }                                                                                            \
  } while (0)
#define CHECK_NEAR(a, b, tol) CHECK(std::fabs((a) - (b)) <= (tol))
