// Isolated-tick spiking network kernels for sm_100a: one fused launch per tick.
//
// Each thread owns one neuron.  It reads and clears its delay-ring slot t%16,
// advances the conductance ALIF state (neurogen/biology.py:132-180 with frozen
// synapses), and the warp ballots its 32 spike bits into one bitmask word.
// The same warp then pushes the outgoing synapses of each of its spiking
// neurons (found by ffs over the ballot mask) into ring slots (t + d) % 16 with
// integer atomics.  Delays are 1..15, so no push of tick t touches slot t%16
// and the kernel boundary orders tick t's deliveries before tick t+1's reads.
//
// Numerics contract (shared with the C oracle, oracle/net_oracle.c): fp32
// state, every operation rounded as written (__f*_rn intrinsics, -fmad=false),
// exp() by the Cody-Waite + degree-7 Taylor scheme below, and the ring holding
// integer multiples of 2^-24 nS so that concurrent deliveries sum exactly,
// independent of order.  Results are bit-identical to the oracle.
#include "net_kernels.h"

#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace ngb {
namespace {

constexpr int TB = 256; // threads per block (8 warps)

__device__ __forceinline__ unsigned long long mix64(unsigned long long z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

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

// Fixed-point amount (2^-24 nS units) and ring component of a signed weight.
__device__ __forceinline__ int quantum(float w) { return __float2int_rn(__fmul_rn(fabsf(w), 16777216.f)); }

__device__ __forceinline__ void deliver(const NetDev &d, long long t, uint32_t word, float w) {
  if (w == 0.f) return;
  const int post = (int)(word & kPostMask);
  const int dly = (int)(word >> 28) + 1;
  const int slot = (int)((t + dly) & (kRingSlots - 1));
  atomicAdd(reinterpret_cast<int *>(d.ring) + ((size_t)slot * d.n + post) * 2 + (w < 0.f ? 1 : 0), quantum(w));
}

__device__ __forceinline__ float half_bits(uint32_t bits16) {
  return __half2float(__ushort_as_half((unsigned short)bits16));
}

// Push all outgoing CSR synapses of `pre` with the whole warp: each lane takes
// 8 consecutive synapses per step (two 16-byte index loads and one 16-byte
// fp16 weight load, or two for fp32), streaming past L1/L2 (evict-first).
__device__ __forceinline__ void push_csr(const NetDev &d, long long t, int pre, int lane) {
  const long long e0 = d.row[pre], e1 = d.row[pre + 1];
  for (long long e = e0 + lane * 8; e < e1; e += 256) {
    const uint4 *ps = reinterpret_cast<const uint4 *>(d.syn + e);
    const uint4 p0 = __ldcs(ps), p1 = __ldcs(ps + 1);
    const uint32_t word[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
    float w[8];
    if (d.w_half) {
      const uint4 wv = __ldcs(reinterpret_cast<const uint4 *>(static_cast<const __half *>(d.w) + e));
      const uint32_t h[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        w[2 * j] = half_bits(h[j] & 0xFFFFu);
        w[2 * j + 1] = half_bits(h[j] >> 16);
      }
    } else {
      const float4 *pw = reinterpret_cast<const float4 *>(static_cast<const float *>(d.w) + e);
      const float4 w0 = __ldcs(pw), w1 = __ldcs(pw + 1);
      w[0] = w0.x; w[1] = w0.y; w[2] = w0.z; w[3] = w0.w;
      w[4] = w1.x; w[5] = w1.y; w[6] = w1.z; w[7] = w1.w;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) deliver(d, t, word[j], w[j]);
  }
}

// Push the spiking columns `sub` (16-bit mask) of block-column bc: each lane
// takes one block, sums the selected tile columns per post row in fixed point
// (E and I apart), and issues one atomic per non-zero row sum.
__device__ __forceinline__ void push_bsr(const NetDev &d, long long t, int bc, unsigned sub, int lane) {
  const long long b0 = d.bcol[bc], b1 = d.bcol[bc + 1];
  for (long long b = b0 + lane; b < b1; b += 32) {
    const uint32_t meta = __ldcs(d.blk + b);
    const int br = (int)(meta & kPostMask);
    const int dly = (int)(meta >> 28) + 1;
    int acc[2][16];
#pragma unroll
    for (int r = 0; r < 16; ++r) acc[0][r] = acc[1][r] = 0;
    unsigned m = sub;
    while (m) {
      const int c = __ffs(m) - 1;
      m &= m - 1;
      const uint4 *col = reinterpret_cast<const uint4 *>(d.tiles + ((size_t)b * 16 + c) * 16);
      const uint4 c0 = __ldcs(col), c1 = __ldcs(col + 1);
      const uint32_t h[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const float w = half_bits(q ? h[j] >> 16 : h[j] & 0xFFFFu);
          const int amount = w == 0.f ? 0 : quantum(w);
          if (w < 0.f) acc[1][2 * j + q] += amount;
          else acc[0][2 * j + q] += amount;
        }
      }
    }
    const int slot = (int)((t + dly) & (kRingSlots - 1));
    int *ring = reinterpret_cast<int *>(d.ring) + ((size_t)slot * d.n + (size_t)br * 16) * 2;
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      if (acc[0][r]) atomicAdd(ring + 2 * r, acc[0][r]);
      if (acc[1][r]) atomicAdd(ring + 2 * r + 1, acc[1][r]);
    }
  }
}

template <bool BSR>
__global__ void __launch_bounds__(TB) k_net_tick(NetDev d, long long t, uint32_t *spikes_out,
                                                 unsigned long long *counts) {
  __shared__ unsigned long long red[2][TB / 32];
  const int i = blockIdx.x * TB + threadIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  bool s = false;
  int events = 0;
  if (i < d.n) {
    const int slot = (int)(t & (kRingSlots - 1));
    int2 *rp = d.ring + (size_t)slot * d.n + i;
    const int2 r = *rp;
    *rp = make_int2(0, 0);
    const bool exc = i < d.n_exc;
    float ge = __fadd_rn(__fmul_rn(d.ge[i], d.dE), __fmul_rn(__int2float_rn(r.x), kRingQuantum));
    const float gi = __fadd_rn(__fmul_rn(d.gi[i], d.dI), __fmul_rn(__int2float_rn(r.y), kRingQuantum));
    const bool ev = drive_event(d, t, i);
    if (d.drive_kind == 0 && ev) ge = __fadd_rn(ge, d.drive_ns);
    float a = __fmul_rn(d.a[i], d.dA);
    const float g = __fadd_rn(__fadd_rn(d.g_leak, ge), gi);
    const float vinf = __fdiv_rn(__fadd_rn(__fsub_rn(__fadd_rn(d.gLEL, __fmul_rn(d.e_inh, gi)), a), d.bias), g);
    const int ref = d.ref[i];
    const bool avail = ref <= 0;
    const float cap = exc ? d.cap_e : d.cap_i;
    const float decay = ng_expf(__fdiv_rn(__fmul_rn(d.neg_dt, g), cap));
    float v = __fadd_rn(vinf, __fmul_rn(__fsub_rn(d.v[i], vinf), decay));
    if (!avail) v = d.v_reset;
    s = d.drive_kind == 1 ? ev : (avail && v >= d.v_th);
    if (s) v = d.v_reset;
    int ref_next = ref > 0 ? ref - 1 : 0;
    if (s) ref_next = d.ref_ticks;
    if (s && exc) a = __fadd_rn(a, d.adapt_inc);
    d.v[i] = v;
    d.a[i] = a;
    d.ge[i] = ge;
    d.gi[i] = gi;
    d.ref[i] = ref_next;
    if (s && counts) events = d.outdeg[i];
  }
  const unsigned fired = __ballot_sync(0xffffffffu, s);
  const int base = i - lane;
  if (spikes_out && lane == 0 && base < d.n) spikes_out[base >> 5] = fired;
  if (BSR) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const unsigned sub = (fired >> (16 * half)) & 0xFFFFu;
      if (sub) push_bsr(d, t, (base >> 4) + half, sub, lane);
    }
  } else {
    unsigned m = fired;
    while (m) {
      const int src = __ffs(m) - 1;
      m &= m - 1;
      push_csr(d, t, base + src, lane);
    }
  }
  if (counts) {
    unsigned long long ev = (unsigned long long)events;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ev += __shfl_down_sync(0xffffffffu, ev, o);
    if (lane == 0) {
      red[0][warp] = __popc(fired);
      red[1][warp] = ev;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long ns = 0, ne = 0;
      for (int k = 0; k < TB / 32; ++k) {
        ns += red[0][k];
        ne += red[1][k];
      }
      if (ns) {
        atomicAdd(counts, ns);
        atomicAdd(counts + 1, ne);
      }
    }
  }
}

} // namespace

void launch_net_tick(const NetDev &d, long long t, uint32_t *spikes_out, unsigned long long *counts,
                     cudaStream_t s) {
  const int blocks = (d.n + TB - 1) / TB;
  if (d.bsr) k_net_tick<true><<<blocks, TB, 0, s>>>(d, t, spikes_out, counts);
  else k_net_tick<false><<<blocks, TB, 0, s>>>(d, t, spikes_out, counts);
}

} // namespace ngb
