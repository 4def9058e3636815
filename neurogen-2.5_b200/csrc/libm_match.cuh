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
    const double inv[17] = {1.0 / 355687428096000.0, 1.0 / 20922789888000.0, 1.0 / 1307674368000.0,
                            1.0 / 87178291200.0, 1.0 / 6227020800.0, 1.0 / 479001600.0, 1.0 / 39916800.0,
                            1.0 / 3628800.0, 1.0 / 362880.0, 1.0 / 40320.0, 1.0 / 5040.0, 1.0 / 720.0,
                            1.0 / 120.0, 1.0 / 24.0, 1.0 / 6.0, 0.5, 1.0};
    for (int i = 0; i < 17; ++i) p = p * x + inv[i];
    return p * x;
  }
  return exp_d(x) - 1.0;
}

// The uncorrected formulas (float arithmetic as written around the double
// exponentials).
NGB_HD float tanh_formula(float x) {
  const float ax = x < 0.f ? -x : x;
  float z;
  if (!(ax < 22.f)) {
    z = 1.f;
  } else if (ax >= 1.f) {
    const float t = float(expm1_d(double(2.f * ax)));
    z = 1.f - 2.f / (t + 2.f);
  } else if (ax < 0x1p-55f) {
    z = ax;
  } else {
    const float t = float(expm1_d(double(-2.f * ax)));
    z = -t / (t + 2.f);
  }
  return x < 0.f ? -z : z;
}
NGB_HD float exp_formula(float x) {
  if (x > 100.f) return float_of(0x7F800000u); // +inf, as float e^x beyond 88.73
  if (x < -110.f) return 0.f;                   // below the smallest subnormal
  return float(exp_d(double(x)));
}
NGB_HD float sigmoid_formula(float x) { return 1.f / (1.f + exp_formula(-x)); }

// Exception table of one function over float inputs with bits in [lo, hi):
// bucket b = (u - lo) >> kShift holds entries[start[b] .. start[b+1]), each
// (u & kLowMask) << 4 | (delta + 8), sorted; delta in -7..7 is the correction
// in ulps (result bits - formula bits).
struct MathTable {
  static constexpr int kShift = 12;
  static constexpr uint32_t kLowMask = (1u << kShift) - 1;
  const uint32_t *start = nullptr;
  const uint16_t *entries = nullptr;
  uint32_t lo = 0, hi = 0;
};

#ifdef __CUDACC__
// Correction (in ulps) of the formula's result at input bits u.
__device__ __forceinline__ int table_delta(const MathTable &t, uint32_t u) {
  if (u < t.lo || u >= t.hi || !t.start) return 0;
  const uint32_t b = (u - t.lo) >> MathTable::kShift;
  int a = (int)__ldg(t.start + b), e = (int)__ldg(t.start + b + 1);
  const uint32_t key = u & MathTable::kLowMask;
  while (a < e) { // first entry with key >= the probe
    const int m = (a + e) >> 1;
    if (((uint32_t)__ldg(t.entries + m) >> 4) < key) a = m + 1;
    else e = m;
  }
  if (a < (int)__ldg(t.start + b + 1)) {
    const uint32_t v = __ldg(t.entries + a);
    if ((v >> 4) == key) return (int)(v & 15u) - 8;
  }
  return 0;
}

// tanhf of the host C library (symmetric in x: the table is keyed by |x|).
__device__ __forceinline__ float tanh_host(float x, const MathTable &t) {
  const float z = tanh_formula(x);
  const int d = table_delta(t, bits_of(x) & 0x7FFFFFFFu);
  if (d == 0) return z;
  const uint32_t zb = bits_of(z);
  return float_of((zb & 0x80000000u) | ((zb & 0x7FFFFFFFu) + (uint32_t)d));
}

// 1 / (1 + expf(-x)) as the host computes it with its C library's expf
// (table keyed by the bits of x, both signs; the result is positive).
__device__ __forceinline__ float sigmoid_host(float x, const MathTable &t) {
  const float z = sigmoid_formula(x);
  const int d = table_delta(t, bits_of(x));
  return d ? float_of(bits_of(z) + (uint32_t)d) : z;
}
#endif

} // namespace libm_match
} // namespace ngb
