// Device tanh and sigmoid that return exactly what the host C library's
// tanhf and expf give (the reference CPU engine calls std::tanh(float) and
// std::exp(float), src/native/NeuralEngine.cpp:9,84-85).
//
// Those functions are not correctly rounded, so no device formula matches
// them on its own.  Instead:
//   1. a formula that is evaluated bit-identically on the host and on the GPU
//      (plain IEEE double arithmetic, no library calls, no contraction: the
//      CUDA files are compiled with -fmad=false and x86-64 host code has no
//      fused multiply-add), accurate to ~1e-16 relative before its final
//      rounding to float;
//   2. a table of the inputs where the host library's result differs from
//      the formula's, built once per process on the host by evaluating both
//      over every float input that can differ, stored as small ulp
//      corrections (math_tables.cpp), uploaded with each model.
// The device result is formula(x) corrected by the table: the host
// library's own value for every input.
//
// tanh uses the expm1 identity tanh|x| = 1 - 2/(e^{2|x|} + 1)
// = 1 - 2/(expm1(2|x|) + 2) for |x| >= 1 and -expm1(-2|x|)/(expm1(-2|x|) + 2)
// below, with tanh x = x for tiny |x| and 1 beyond 22 (the saturation of
// fp32); sigmoid(x) = 1 / (1 + e^{-x}) in float, its table holding the
// corrections of the final quotient.
#pragma once
#include <cstdint>

#ifdef __CUDACC__
#define NGB_HD __host__ __device__ __forceinline__
#else
#define NGB_HD inline
#endif

namespace ngb {
namespace libm_match {

NGB_HD uint32_t bits_of(float f) {
#ifdef __CUDA_ARCH__
  return __float_as_uint(f);
#else
  uint32_t u;
  __builtin_memcpy(&u, &f, 4);
  return u;
#endif
}
NGB_HD float float_of(uint32_t u) {
#ifdef __CUDA_ARCH__
  return __uint_as_float(u);
#else
  float f;
  __builtin_memcpy(&f, &u, 4);
  return f;
#endif
}
NGB_HD double pow2(int k) { // 2^k for -1022 <= k <= 1023
  const uint64_t u = uint64_t(k + 1023) << 52;
#ifdef __CUDA_ARCH__
  return __longlong_as_double((long long)u);
#else
  double d;
  __builtin_memcpy(&d, &u, 8);
  return d;
#endif
}

// e^x for -700 < x < 700: x = k ln2 + r (ln2 in two parts, the high part
// with trailing zero bits so k * high is exact), e^r by its Taylor series to
// degree 13 (|r| <= 0.35: truncation below 1e-18), scaled by 2^k.
NGB_HD double exp_d(double x) {
  const double kd = x * 1.4426950408889634;
  const double kr = kd >= 0 ? double((long long)(kd + 0.5)) : -double((long long)(-kd + 0.5));
  const double r = (x - kr * 0.693147180369123816490) - kr * 1.90821492927058770002e-10;
  double p = 1.0 / 6227020800.0; // 1/13!
  p = p * r + 1.0 / 479001600.0;
  p = p * r + 1.0 / 39916800.0;
  p = p * r + 1.0 / 3628800.0;
  p = p * r + 1.0 / 362880.0;
  p = p * r + 1.0 / 40320.0;
  p = p * r + 1.0 / 5040.0;
  p = p * r + 1.0 / 720.0;
  p = p * r + 1.0 / 120.0;
  p = p * r + 1.0 / 24.0;
  p = p * r + 1.0 / 6.0;
  p = p * r + 0.5;
  p = p * r + 1.0;
  p = p * r + 1.0;
  return p * pow2(int(kr));
}

// e^x - 1: Taylor series for |x| < 0.5 (degree 18, truncation below 1e-20
// relative), exp_d(x) - 1 otherwise.
NGB_HD double expm1_d(double x) {
  if (x > -0.5 && x < 0.5) {
    double p = 1.0 / 6402373705728000.0; // 1/18!
    p = p * x + 1.0 / 355687428096000.0;
    p = p * x + 1.0 / 20922789888000.0;
    p = p * x + 1.0 / 1307674368000.0;
    p = p * x + 1.0 / 87178291200.0;
    p = p * x + 1.0 / 6227020800.0;
    p = p * x + 1.0 / 479001600.0;
    p = p * x + 1.0 / 39916800.0;
    p = p * x + 1.0 / 3628800.0;
    p = p * x + 1.0 / 362880.0;
    p = p * x + 1.0 / 40320.0;
    p = p * x + 1.0 / 5040.0;
    p = p * x + 1.0 / 720.0;
    p = p * x + 1.0 / 120.0;
    p = p * x + 1.0 / 24.0;
    p = p * x + 1.0 / 6.0;
    p = p * x + 0.5;
    p = p * x + 1.0;
    return p * x;
  }
  return exp_d(x) - 1.0;
}

// The uncorrected formulas (float arithmetic as written around the double
// exponentials).  The *_d forms also return the double value that was
// rounded to float (the exponential), or 0 where none was.
NGB_HD float tanh_formula_d(float x, double &e) {
  const float ax = x < 0.f ? -x : x;
  float z;
  e = 0.0;
  if (!(ax < 22.f)) {
    z = 1.f;
  } else if (ax >= 1.f) {
    e = expm1_d(double(2.f * ax));
    const float t = float(e);
    z = 1.f - 2.f / (t + 2.f);
  } else if (ax < 0x1p-55f) {
    z = ax;
  } else {
    e = expm1_d(double(-2.f * ax));
    const float t = float(e);
    z = -t / (t + 2.f);
  }
  return x < 0.f ? -z : z;
}
NGB_HD float tanh_formula(float x) {
  double e;
  return tanh_formula_d(x, e);
}
NGB_HD float exp_formula_d(float x, double &e) {
  e = 0.0;
  if (x > 100.f) return float_of(0x7F800000u); // +inf, as float e^x beyond 88.73
  if (x < -110.f) return 0.f;                   // below the smallest subnormal
  e = exp_d(double(x));
  return float(e);
}
NGB_HD float exp_formula(float x) {
  double e;
  return exp_formula_d(x, e);
}
NGB_HD float sigmoid_formula_d(float x, double &e) { return 1.f / (1.f + exp_formula_d(-x, e)); }
NGB_HD float sigmoid_formula(float x) {
  double e;
  return sigmoid_formula_d(x, e);
}

// Distance, in ulps of the float it rounds to, from a double value to the
// nearest rounding midpoint between two floats (0: on a midpoint; 0.5: on a
// float).  Exact power-of-two scalings only, so host and device agree.  A
// library's float function can round differently from the correctly rounded
// value only near a midpoint; the tables record, per function, the largest
// distance at which the library differs from the formula, and inputs farther
// out need no lookup.
NGB_HD double midpoint_distance(double e) {
  const float f = float(e);
  const uint32_t fb = bits_of(f) & 0x7FFFFFFFu;
  if (e == 0.0 || fb >= 0x7F800000u) return 0.5;
  const int ex = int(fb >> 23);
  const double r = (e - double(f)) * pow2(149 - (ex ? ex - 1 : 0)); // residual in ulps
  return 0.5 - (r < 0 ? -r : r);
}

// Exception table of one function over float inputs with bits in [lo, hi):
// bucket b = (u - lo) >> shift holds entries[start[b] .. start[b+1]), each
// (u & (2^shift - 1)) << 4 | (delta + 8), sorted; delta in -7..7 is the
// correction in ulps (result bits - formula bits).  shift <= 12 (16-bit
// entries); steps = ceil(log2(largest bucket + 1)) bounds the search.
// An input whose formula intermediate lies farther than skip[exponent of the
// input] from a midpoint needs no lookup (a negative threshold: no lookup at
// all).  Optionally a dense map of 3-bit codes for the inputs in
// [map_lo, map_hi) (10 a word: delta + 3 for delta in -3..3, 7 look in the
// buckets) answers a lookup in one load.
struct MathTable {
  const uint32_t *start = nullptr;
  const uint16_t *entries = nullptr;
  uint32_t lo = 0, hi = 0;
  int shift = 8, steps = 0;
  const float *skip = nullptr; // [256]
  const uint32_t *map = nullptr;
  uint32_t map_lo = 0, map_hi = 0;
};

#ifdef __CUDACC__
// Code of input u in the table's dense map: the correction + 3, or 7 to look
// in the buckets (also for inputs outside the map).
__device__ __forceinline__ uint32_t map_code(const MathTable &t, uint32_t u) {
  if (!t.map || u < t.map_lo || u >= t.map_hi) return 7u;
  const uint32_t i = u - t.map_lo, w = i / 10u;
  return (__ldg(t.map + w) >> (3u * (i - 10u * w))) & 7u;
}

// Whether input u, whose formula intermediate is e, can need a correction.
__device__ __forceinline__ bool near_midpoint(const MathTable &t, uint32_t u, double e) {
  const float th = __ldg(t.skip + (u >> 23));
  return th >= 0.f && midpoint_distance(e) <= (double)th;
}

// Bucket search for input bits u: the correction, or 0.
__device__ __forceinline__ int bucket_delta(const MathTable &t, uint32_t u) {
  if (u < t.lo || u >= t.hi) return 0;
  const uint32_t b = (u - t.lo) >> t.shift;
  const int a = (int)__ldg(t.start + b), e = (int)__ldg(t.start + b + 1);
  if (a == e) return 0;
  const uint32_t key = u & ((1u << t.shift) - 1u);
  int first = a, len = e - a;
#pragma unroll 1
  for (int i = 0; i < 13; ++i) {
    if (i < t.steps && len > 0) {
      const int half = len >> 1;
      if (((uint32_t)__ldg(t.entries + first + half) >> 4) < key) {
        first += half + 1;
        len -= half + 1;
      } else {
        len = half;
      }
    }
  }
  if (first < e) {
    const uint32_t v = __ldg(t.entries + first);
    if ((v >> 4) == key) return (int)(v & 15u) - 8;
  }
  return 0;
}

// Correction (in ulps) of the formula's result at input bits u, given the
// formula's double intermediate e.
__device__ __forceinline__ int table_delta(const MathTable &t, uint32_t u, double e) {
  if (!near_midpoint(t, u, e)) return 0;
  const uint32_t code = map_code(t, u);
  if (code != 7u) return (int)code - 3;
  return bucket_delta(t, u);
}

// Corrections of N independent inputs: key u[s] (with formula intermediate
// e[s]) in table which[s] of (t0, t1, t2), none when which[s] < 0.  The map
// loads of all N are issued together; the rare bucket searches follow one at
// a time (a rolled loop keeps the code small).  Tables are selected by index,
// not pointer, so kernel parameters stay in place.
template <int N>
__device__ __forceinline__ void table_deltas(const MathTable &t0, const MathTable &t1, const MathTable &t2,
                                             const int (&which)[N], const uint32_t (&u)[N], const double (&e)[N],
                                             int (&d)[N]) {
  bool search[N];
#pragma unroll
  for (int s = 0; s < N; ++s) {
    const int w = which[s];
    const MathTable &t = w == 0 ? t0 : w == 1 ? t1 : t2;
    d[s] = 0;
    search[s] = false;
    if (w >= 0 && near_midpoint(t, u[s], e[s])) {
      const uint32_t code = map_code(t, u[s]);
      if (code == 7u) search[s] = true;
      else d[s] = (int)code - 3;
    }
  }
  bool any = false;
#pragma unroll
  for (int s = 0; s < N; ++s) any = any || search[s];
  if (any) {
    int dd[N];
    uint32_t uu[N];
    int ww[N];
    bool ss[N];
#pragma unroll
    for (int s = 0; s < N; ++s) dd[s] = 0, uu[s] = u[s], ww[s] = which[s], ss[s] = search[s];
#pragma unroll 1
    for (int s = 0; s < N; ++s)
      if (ss[s]) dd[s] = bucket_delta(ww[s] == 0 ? t0 : ww[s] == 1 ? t1 : t2, uu[s]);
#pragma unroll
    for (int s = 0; s < N; ++s)
      if (search[s]) d[s] = dd[s];
  }
}

// Apply a correction of d ulps to a result's magnitude.
__device__ __forceinline__ float add_ulps(float z, int d) {
  if (d == 0) return z;
  const uint32_t zb = bits_of(z);
  return float_of((zb & 0x80000000u) | ((zb & 0x7FFFFFFFu) + (uint32_t)d));
}

// tanhf of the host C library (symmetric in x: the table is keyed by |x|).
__device__ __forceinline__ float tanh_host(float x, const MathTable &t) {
  double e;
  const float z = tanh_formula_d(x, e);
  return add_ulps(z, table_delta(t, bits_of(x) & 0x7FFFFFFFu, e));
}

// 1 / (1 + expf(-x)) as the host computes it with its C library's expf: one
// table for x >= 0 and one for x < 0, each keyed by |x| (the result is
// positive).
__device__ __forceinline__ float sigmoid_host(float x, const MathTable &pos, const MathTable &neg) {
  double e;
  const float z = sigmoid_formula_d(x, e);
  const uint32_t u = bits_of(x);
  return add_ulps(z, table_delta((u >> 31) ? neg : pos, u & 0x7FFFFFFFu, e));
}
#endif

} // namespace libm_match
} // namespace ngb
