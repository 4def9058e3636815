// Fixed fan-in synapses generated on the device, for neuron-partitioned
// networks (each rank draws only the synapses onto the neurons it holds).
//
// The draws are the host generator's (net_engine.cpp generate_csr): held post
// j takes `fanin` presynaptic cells keyed (j, k) from the counter-based
// splitmix64 streams, a delay and an |N(0, sigma)| fp16 weight (Box-Muller in
// double) signed by the presynaptic cell's type.  Rows come out in the same
// padded layout (delay-1 synapses first, each segment padded to 8), with the
// synapses inside a segment in arrival order of the atomic cursors: the order
// differs from run to run, the network and every result do not (the delay ring
// sums integers).  The double log/cos here are CUDA's where the host uses
// glibc's; a weight can differ only when sigma*z lies within one double ulp of
// an fp32 and then fp16 rounding boundary.
#include "net_kernels.h"

#include <cuda_fp16.h>

namespace ngb {
namespace {

__device__ __forceinline__ unsigned long long mix64(unsigned long long z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__device__ __forceinline__ unsigned long long bits(unsigned long long key, unsigned long long a, unsigned long long b) {
  return mix64(((a << 32) | (b & 0xFFFFFFFFull)) ^ key);
}

// Uniform integer in [0, m): the high 64 bits of bits * m.
__device__ __forceinline__ unsigned long long below(unsigned long long key, unsigned long long a, unsigned long long b,
                                                    unsigned long long m) {
  return __umul64hi(bits(key, a, b), m);
}

__device__ __forceinline__ int draw_pre(const FaninGen &g, int j, int k) {
  const int pre = (int)below(g.key_pre, (unsigned)j, (unsigned)k, (unsigned long long)g.n);
  return pre == j ? (pre + 1) % g.n : pre;
}

__device__ __forceinline__ int draw_delay(const FaninGen &g, int j, int k) {
  return g.delay_min + (int)below(g.key_delay, (unsigned)j, (unsigned)k, (unsigned long long)g.delay_span);
}

// fp16 bits of |N(0, sigma)| keyed (j, k), sign bit set for inhibitory cells.
__device__ __forceinline__ uint16_t draw_weight(const FaninGen &g, int j, int k, bool inhibitory) {
  const double u1 = (double)((bits(g.key_w1, (unsigned)j, (unsigned)k) >> 11) + 1) * 0x1.0p-53; // (0, 1]
  const double u2 = (double)(bits(g.key_w2, (unsigned)j, (unsigned)k) >> 11) * 0x1.0p-53;
  const double z = sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
  const float m = (float)fabs((double)g.sigma * z);
  __half h = __float2half_rn(m);
  if (__half2float(h) == 0.f) h = __ushort_as_half((unsigned short)1); // smallest subnormal, 2^-24
  uint16_t b = __half_as_ushort(h);
  if (inhibitory) b |= 0x8000u;
  return b;
}

// Thread per held post: count its synapses per presynaptic row, delay-1 apart.
__global__ void k_fanin_count(FaninGen g, int *c1, int *c2) {
  const int jl = blockIdx.x * blockDim.x + threadIdx.x;
  if (jl >= g.np) return;
  const int j = g.lo + jl;
  for (int k = 0; k < g.fanin; ++k) {
    const int pre = draw_pre(g, j, k);
    atomicAdd(draw_delay(g, j, k) == 1 ? c1 + pre : c2 + pre, 1);
  }
}

// Thread per held post: place its synapses through the rows' cursors and check
// that its summed input per sign stays inside the ring's fixed-point range
// (the lowest failing post is reported).
__global__ void k_fanin_fill(FaninGen g, const long long *row, const int *mid, int *cur1, int *cur2, uint32_t *syn,
                             uint16_t *w16, int *bad_post) {
  const int jl = blockIdx.x * blockDim.x + threadIdx.x;
  if (jl >= g.np) return;
  const int j = g.lo + jl;
  double sum_e = 0.0, sum_i = 0.0;
  for (int k = 0; k < g.fanin; ++k) {
    const int pre = draw_pre(g, j, k);
    const int d = draw_delay(g, j, k);
    const uint16_t hb = draw_weight(g, j, k, pre >= g.n_exc);
    const long long e = d == 1 ? row[pre] + atomicAdd(cur1 + pre, 1) : row[pre] + mid[pre] + atomicAdd(cur2 + pre, 1);
    syn[e] = (uint32_t)jl | ((uint32_t)(d - 1) << 28);
    w16[e] = hb;
    const double w = (double)__half2float(__ushort_as_half(hb));
    if (w < 0) sum_i += fabs(w);
    else sum_e += fabs(w);
  }
  if (sum_e >= 127.0 || sum_i >= 127.0) atomicMin(bad_post, jl);
}

} // namespace

void launch_fanin_count(const FaninGen &g, int *c1, int *c2, cudaStream_t s) {
  if (g.np > 0) k_fanin_count<<<(g.np + 255) / 256, 256, 0, s>>>(g, c1, c2);
}

void launch_fanin_fill(const FaninGen &g, const long long *row, const int *mid, int *cur1, int *cur2, uint32_t *syn,
                       uint16_t *w16, int *bad_post, cudaStream_t s) {
  if (g.np > 0) k_fanin_fill<<<(g.np + 255) / 256, 256, 0, s>>>(g, row, mid, cur1, cur2, syn, w16, bad_post);
}

} // namespace ngb
