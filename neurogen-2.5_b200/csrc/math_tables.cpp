// Exception tables of tanh and sigmoid: every float input where the host C
// library's result (tanhf; 1 / (1 + expf(-x))) differs from the formula the
// device evaluates (libm_match.cuh), with the difference in ulps.
//
// Covered inputs: tanh over |x| in [2^-40, 22) (below, both give x; beyond,
// both give 1), sigmoid over x in [-88.8, 16.75] minus |x| < 2^-40 (beyond
// -88.8 both give 0; beyond 16.75 both give 1, since e^{-x} is then below half
// an ulp of 1; for tiny |x| both give exactly 0.5).  Built in parallel over
// fixed bucket ranges, so the table does not depend on the thread count.
#include "math_tables.h"

#include <cmath>
#include <mutex>
#include <stdexcept>
#include <string>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace ngb {
namespace {
using namespace libm_match;

template <class Ref, class Formula>
void build(HostMathTable &t, uint32_t lo, uint32_t hi, Ref ref, Formula formula) {
  constexpr int S = MathTable::kShift;
  t.lo = lo & ~MathTable::kLowMask;
  const uint32_t buckets = ((hi - t.lo) >> S) + 1;
  t.hi = t.lo + (buckets << S);
  std::vector<std::vector<uint16_t>> per(buckets);
  int bad = 0;
#pragma omp parallel for schedule(dynamic, 64) reduction(| : bad)
  for (long long b = 0; b < (long long)buckets; ++b) {
    const uint32_t u0 = t.lo + (uint32_t(b) << S);
    for (uint32_t k = 0; k <= MathTable::kLowMask; ++k) {
      const uint32_t u = u0 + k;
      if (u < lo || u >= hi) continue;
      const float x = float_of(u);
      const int64_t d = int64_t(bits_of(ref(x))) - int64_t(bits_of(formula(x)));
      if (d == 0) continue;
      if (d < -7 || d > 7) {
        bad = 1;
        continue;
      }
      per[b].push_back(uint16_t((k << 4) | uint32_t(d + 8)));
    }
  }
  if (bad) throw std::runtime_error("host math library differs from the device formula by more than 7 ulps");
  t.start.assign(size_t(buckets) + 1, 0);
  size_t total = 0;
  for (uint32_t b = 0; b < buckets; ++b) {
    t.start[b] = uint32_t(total);
    total += per[b].size();
  }
  t.start[buckets] = uint32_t(total);
  t.entries.reserve(total);
  for (auto &v : per) t.entries.insert(t.entries.end(), v.begin(), v.end());
}
} // namespace

const HostMathTable &tanh_table() {
  static HostMathTable t;
  static std::once_flag once;
  std::call_once(once, [] {
    build(t, bits_of(0x1p-40f), bits_of(22.f), [](float x) { return std::tanh(x); },
          [](float x) { return tanh_formula(x); });
  });
  return t;
}

const HostMathTable &sigmoid_table() {
  static HostMathTable t;
  static std::once_flag once;
  std::call_once(once, [] {
    HostMathTable pos, neg;
    auto ref = [](float x) { return 1.f / (1.f + std::exp(-x)); };
    auto formula = [](float x) { return sigmoid_formula(x); };
    // Positive inputs [2^-40, 16.75], then negative ones (bit 31 set) up to -88.8.
    build(pos, bits_of(0x1p-40f), bits_of(16.75f) + 1, ref, formula);
    build(neg, bits_of(-0x1p-40f), bits_of(-88.8f) + 1, ref, formula);
    // One table over [pos.lo, neg.hi): the unsigned keys between the two
    // ranges (positive floats above 16.75, negative ones below 2^-40 in
    // magnitude) have no entries.
    t.lo = pos.lo;
    t.hi = neg.hi;
    const uint32_t buckets = (t.hi - t.lo) >> MathTable::kShift;
    t.start.assign(size_t(buckets) + 1, 0);
    const uint32_t pos_b = (pos.hi - pos.lo) >> MathTable::kShift, neg_b0 = (neg.lo - t.lo) >> MathTable::kShift;
    t.entries = pos.entries;
    for (uint32_t b = 0; b <= buckets; ++b) {
      if (b <= pos_b) t.start[b] = pos.start[b];
      else if (b < neg_b0) t.start[b] = uint32_t(pos.entries.size());
      else t.start[b] = uint32_t(pos.entries.size()) + neg.start[b - neg_b0];
    }
    t.entries.insert(t.entries.end(), neg.entries.begin(), neg.entries.end());
  });
  return t;
}

} // namespace ngb
