// Device arithmetic shared by the isolated-tick network kernels
// (net_kernels.cu: per-tick launches; net_resident.cu: persistent launch).
//
// Numerics contract (shared with the C oracle, oracle/net_oracle.c): fp32
// state, every operation rounded as written (__f*_rn intrinsics, -fmad=false),
// exp() by the Cody-Waite + degree-7 Taylor scheme below, and the delay ring
// holding integer multiples of 2^-24 nS so that concurrent deliveries sum
// exactly, independent of order.  Both kernels are bit-identical to the oracle.
#pragma once
#include "net_kernels.h"

#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace ngb {
namespace netdev {

__device__ __forceinline__ long long tick_of(const TickRef &r) { return r.t_dev ? *r.t_dev + r.k : r.k; }

__device__ __forceinline__ unsigned long long mix64(unsigned long long z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// External drive draw of global neuron i at tick t (counter-based hash).
__device__ __forceinline__ bool drive_event(const NetDev &d, long long t, int i) {
  const unsigned long long key = ((unsigned long long)t << 32) | (unsigned)i;
  return (unsigned)(mix64(key ^ d.drive_key) >> 32) < d.drive_thr;
}

// exp(x), x <= 0: Cody-Waite reduction x = k ln2 + r (15-bit head of ln2 so
// k*head is exact), e^r by its degree-7 Taylor polynomial, scale by 2^k.
__device__ __forceinline__ float ng_expf(float x) {
  if (x < -87.f) return 0.f;
  const float kf = rintf(__fmul_rn(x, 1.44269504f));
  const float r = __fsub_rn(__fsub_rn(x, __fmul_rn(kf, 0.693145751953125f)), __fmul_rn(kf, 1.42860682e-06f));
  float p = 0.000198412701f;
  p = __fadd_rn(__fmul_rn(p, r), 0.00138888892f);
  p = __fadd_rn(__fmul_rn(p, r), 0.00833333377f);
  p = __fadd_rn(__fmul_rn(p, r), 0.0416666679f);
  p = __fadd_rn(__fmul_rn(p, r), 0.166666672f);
  p = __fadd_rn(__fmul_rn(p, r), 0.5f);
  p = __fadd_rn(__fmul_rn(p, r), 1.0f);
  p = __fadd_rn(__fmul_rn(p, r), 1.0f);
  const int k = (int)kf;
  if (k >= -126) return __fmul_rn(p, __int_as_float((127 + k) << 23));
  return __fmul_rn(__fmul_rn(p, __int_as_float((127 + k + 64) << 23)), 5.42101086e-20f);
}

// Membrane, conductance, adaptation and refractory update of global neuron
// gidx at tick t, given the ring arrivals r (E, I) for this tick, in the
// operation order of the oracle's on_run.  Updates the state in place and
// returns the spike.
__device__ __forceinline__ bool alif_math(const NetDev &d, long long t, int gidx, int2 r, float &v_io, float &a_io,
                                          float &ge_io, float &gi_io, int &ref_io) {
  const bool exc = gidx < d.n_exc;
  float ge = __fadd_rn(__fmul_rn(ge_io, d.dE), __fmul_rn(__int2float_rn(r.x), kRingQuantum));
  const float gi = __fadd_rn(__fmul_rn(gi_io, d.dI), __fmul_rn(__int2float_rn(r.y), kRingQuantum));
  const bool ev = drive_event(d, t, gidx);
  if (d.drive_kind == 0 && ev) ge = __fadd_rn(ge, d.drive_ns);
  float a = __fmul_rn(a_io, d.dA);
  const float g = __fadd_rn(__fadd_rn(d.g_leak, ge), gi);
  const float vinf = __fdiv_rn(__fadd_rn(__fsub_rn(__fadd_rn(d.gLEL, __fmul_rn(d.e_inh, gi)), a), d.bias), g);
  const int ref = ref_io;
  const bool avail = ref <= 0;
  const float cap = exc ? d.cap_e : d.cap_i;
  const float decay = ng_expf(__fdiv_rn(__fmul_rn(d.neg_dt, g), cap));
  float v = __fadd_rn(vinf, __fmul_rn(__fsub_rn(v_io, vinf), decay));
  if (!avail) v = d.v_reset;
  const bool s = d.drive_kind == 1 ? ev : (avail && v >= d.v_th);
  if (s) v = d.v_reset;
  int ref_next = ref > 0 ? ref - 1 : 0;
  if (s) ref_next = d.ref_ticks;
  if (s && exc) a = __fadd_rn(a, d.adapt_inc);
  v_io = v;
  a_io = a;
  ge_io = ge;
  gi_io = gi;
  ref_io = ref_next;
  return s;
}

// Fixed-point amount (2^-24 nS units) of a signed weight.
__device__ __forceinline__ int quantum(float w) { return __float2int_rn(__fmul_rn(fabsf(w), 16777216.f)); }

__device__ __forceinline__ float half_bits(uint32_t bits16) {
  return __half2float(__ushort_as_half((unsigned short)bits16));
}

} // namespace netdev
} // namespace ngb
