// Exception tables of tanh and sigmoid: every float input where the host C
// library's result (tanhf; 1 / (1 + expf(-x))) differs from the formula the
// device evaluates (libm_match.cuh), with the difference in ulps.
//
// Scanned inputs: tanh over |x| in [2^-40, 22) (below, both give x; beyond,
// both give 1); sigmoid over x in [2^-40, 16.75] and [-88.8, -2^-40] (beyond
// -88.8 both give 0; beyond 16.75 both give 1, e^{-x} being under half an ulp
// of 1; for |x| < 2^-40 both give exactly 0.5).  The stored range is trimmed
// to the buckets that hold entries.  Built in parallel over fixed bucket
// ranges, so the tables do not depend on the thread count.
#include "math_tables.h"

#include <algorithm>
#include <cmath>
#include <mutex>
#include <stdexcept>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace ngb {
namespace {
using namespace libm_match;

// Entries of the inputs u in [lo, hi) (float bits) where ref differs from
// formula, in buckets of 2^shift inputs.
// formula(x, e) returns the device formula's result and its double
// intermediate e; the table's skip threshold is the largest midpoint distance
// of e over the entries.
template <class Ref, class Formula>
void build(HostMathTable &t, uint32_t lo, uint32_t hi, int shift, Ref ref, Formula formula) {
  const uint32_t mask = (1u << shift) - 1u;
  const uint32_t base = lo & ~mask;
  const uint32_t buckets = ((hi - 1 - base) >> shift) + 1;
  std::vector<std::vector<uint16_t>> per(buckets);
  std::vector<std::vector<double>> far(buckets); // midpoint distance of each entry
  int bad = 0;
#pragma omp parallel for schedule(dynamic, 256) reduction(| : bad)
  for (long long b = 0; b < (long long)buckets; ++b) {
    const uint32_t u0 = base + (uint32_t(b) << shift);
    for (uint32_t k = 0; k <= mask; ++k) {
      const uint32_t u = u0 + k;
      if (u < lo || u >= hi) continue;
      const float x = float_of(u);
      double e;
      const float z = formula(x, e);
      const int64_t d = int64_t(bits_of(ref(x))) - int64_t(bits_of(z));
      if (d == 0) continue;
      if (d < -7 || d > 7) {
        bad = 1;
        continue;
      }
      far[b].push_back(midpoint_distance(e));
      per[b].push_back(uint16_t((k << 4) | uint32_t(d + 8)));
    }
  }
  if (bad) throw std::runtime_error("host math library differs from the device formula by more than 7 ulps");
  // Skip thresholds per exponent of the input, rounded up to float.
  std::vector<double> th(256, -1.0);
  for (uint32_t b = 0; b < buckets; ++b)
    for (size_t i = 0; i < per[b].size(); ++i) {
      const uint32_t u = base + (b << shift) + (uint32_t(per[b][i]) >> 4);
      th[u >> 23] = std::max(th[u >> 23], far[b][i]);
    }
  for (int x = 0; x < 256; ++x) {
    float f = float(th[x]);
    if (double(f) < th[x]) f = std::nextafter(f, 1.f);
    t.skip[x] = th[x] < 0 ? -1.f : f;
  }
  // Trim to the buckets that hold entries.
  uint32_t b0 = 0, b1 = buckets;
  while (b0 < b1 && per[b0].empty()) ++b0;
  while (b1 > b0 && per[b1 - 1].empty()) --b1;
  t.shift = shift;
  t.lo = base + (b0 << shift);
  t.hi = base + (b1 << shift);
  t.start.assign(size_t(b1 - b0) + 1, 0);
  size_t total = 0, largest = 0;
  for (uint32_t b = b0; b < b1; ++b) {
    t.start[b - b0] = uint32_t(total);
    total += per[b].size();
    largest = std::max(largest, per[b].size());
  }
  t.start[b1 - b0] = uint32_t(total);
  t.entries.clear();
  t.entries.reserve(total);
  for (uint32_t b = b0; b < b1; ++b) t.entries.insert(t.entries.end(), per[b].begin(), per[b].end());
  t.steps = 0;
  while ((size_t(1) << t.steps) <= largest) ++t.steps;
  if (t.steps > 13) throw std::logic_error("math table bucket too large");
}

// Dense 3-bit codes of the inputs [lo, hi) from the table's entries: the
// correction + 3 (3: none), or 7 for a correction beyond +-3 ulps (looked up
// in the buckets).
void build_map(HostMathTable &t, uint32_t lo, uint32_t hi) {
  t.map_lo = lo;
  t.map_hi = hi;
  const uint32_t n = hi - lo;
  t.map.assign(size_t(n + 9) / 10, 0u);
  for (uint32_t i = 0; i < n; ++i) t.map[i / 10] |= 3u << (3 * (i % 10)); // no correction
  const uint32_t nb = uint32_t(t.start.size() - 1);
  for (uint32_t b = 0; b < nb; ++b)
    for (uint32_t i = t.start[b]; i < t.start[b + 1]; ++i) {
      const uint32_t u = t.lo + (b << t.shift) + (uint32_t(t.entries[i]) >> 4);
      if (u < lo || u >= hi) continue;
      const int d = int(t.entries[i] & 15u) - 8;
      const uint32_t code = (d >= -3 && d <= 3) ? uint32_t(d + 3) : 7u, j = u - lo;
      t.map[j / 10] = (t.map[j / 10] & ~(7u << (3 * (j % 10)))) | (code << (3 * (j % 10)));
    }
}

float sigmoid_ref(float x) { return 1.f / (1.f + std::exp(-x)); }
} // namespace

const HostMathTable &tanh_table() {
  static HostMathTable t;
  static std::once_flag once;
  std::call_once(once, [] {
    build(t, bits_of(0x1p-40f), bits_of(22.f), 8, [](float x) { return std::tanh(x); },
          [](float x, double &e) { return tanh_formula_d(x, e); });
    // Nearly all entries lie in [2^-8, 8): a dense map there (37 MB).
    build_map(t, bits_of(0x1p-8f), bits_of(8.f));
  });
  return t;
}

const HostMathTable &sigmoid_table(bool negative) {
  static HostMathTable t[2];
  static std::once_flag once;
  std::call_once(once, [] {
    build(t[0], bits_of(0x1p-40f), bits_of(16.75f) + 1, 12, [](float x) { return sigmoid_ref(x); },
          [](float x, double &e) { return sigmoid_formula_d(x, e); });
    // Negative inputs, keyed by |x|.
    build(t[1], bits_of(0x1p-40f), bits_of(88.8f) + 1, 12, [](float a) { return sigmoid_ref(-a); },
          [](float a, double &e) { return sigmoid_formula_d(-a, e); });
  });
  return t[negative ? 1 : 0];
}

} // namespace ngb
