// checker.h — element-wise closeness check of the host harness. Same API and rule
// as the reference's include/common/checker.h:10-61 (DefaultTol, CheckReport,
// check_close: count of |g - e| > atol + rtol*|e|, print_report) plus the norm-wise
// relative error this build also reports.
#pragma once

#include <cmath>
#include <cstdio>
#include <vector>

namespace hopper {

template <typename T>
struct DefaultTol {
  static constexpr double rtol = 1e-5;
  static constexpr double atol = 1e-6;
};
template <>
struct DefaultTol<float> {
  static constexpr double rtol = 2e-5;
  static constexpr double atol = 1e-6;
};

struct CheckReport {
  bool pass = false;
  size_t n = 0;
  size_t mismatches = 0;
  double max_abs_err = 0.0;
  double max_rel_err = 0.0;
};

template <typename T>
CheckReport check_close(const std::vector<T>& got, const std::vector<T>& ref, double rtol,
                        double atol) {
  CheckReport r;
  r.n = got.size();
  if (got.size() != ref.size()) {  // size mismatch: every element counts as a failure
    r.mismatches = r.n;
    return r;
  }
  for (size_t i = 0; i < r.n; ++i) {
    const double g = double(got[i]), e = double(ref[i]);
    const double d = std::fabs(g - e);
    const double rel = d / std::fmax(std::fabs(e), 1e-30);
    r.max_abs_err = d > r.max_abs_err ? d : r.max_abs_err;
    r.max_rel_err = rel > r.max_rel_err ? rel : r.max_rel_err;
    if (d > atol + rtol * std::fabs(e)) ++r.mismatches;
  }
  r.pass = r.mismatches == 0;
  return r;
}

template <typename T>
CheckReport check_close(const std::vector<T>& got, const std::vector<T>& ref) {
  return check_close(got, ref, DefaultTol<T>::rtol, DefaultTol<T>::atol);
}

// ||got - ref||_F / ||ref||_F (the BASELINE relative-error measure).
template <typename T>
double norm_rel_error(const std::vector<T>& got, const std::vector<T>& ref) {
  double num = 0.0, den = 0.0;
  for (size_t i = 0; i < got.size() && i < ref.size(); ++i) {
    const double d = double(got[i]) - double(ref[i]);
    num += d * d;
    den += double(ref[i]) * double(ref[i]);
  }
  return den > 0.0 ? std::sqrt(num / den) : std::sqrt(num);
}

inline void print_report(const CheckReport& r, const char* tag) {
  std::printf("[CHECK ] %-20s : %s  (n=%zu mismatch=%zu max_abs=%.3e max_rel=%.3e)\n", tag,
              r.pass ? "PASS" : "FAIL", r.n, r.mismatches, r.max_abs_err, r.max_rel_err);
}

}  // namespace hopper
