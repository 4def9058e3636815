// Resident tick: one persistent cooperative launch runs many ticks of an
// unpartitioned network with the neuron state and the delay ring held in
// shared memory.
//
// CTA c owns neurons [c*P, c*P + P).  Their V, adaptation, g_E, g_I and
// refractory counters, and a ring of Dr slots (Dr = the largest delay rounded
// up to a power of two) of (E, I) fixed-point arrivals, stay in shared memory
// for the whole launch.  Synapses are re-laid out once, at network creation,
// as owner blocks: for presynaptic neuron p and owner CTA c, one block of 8
// event words holding p's synapses onto c's neurons, with a link to overflow
// blocks when p has more than 8 synapses there.  The shared ring is laid out
// [slot][E, I][post]; an event word carries its ring offset for tick 0,
// 2*d*P + (P if inhibitory) + post, and the weight
// (fp16 magnitude, or the precomputed fixed-point amount for fp32 weights), so
// a delivery is one add, one unsigned min and one shared-memory atomic.
//
// A tick is
//   1. membrane update of the CTA's own neurons from its shared ring slot
//      (two neurons a thread when the CTA holds more neurons than threads);
//   2. the CTA reserves a range of this tick's global spike list with one
//      atomic (counters rotate over three ticks) and writes its spike ids;
//   3. one grid barrier (bounded wait), after which the list is complete;
//   4. each warp takes rounds of 32 list entries: each lane loads the owner
//      block (p, c) of one spike (the next two rounds' blocks stay in flight
//      while it delivers one) and delivers its 8 slots with predicated
//      shared-memory atomics.  A warp delivers the overflow blocks it met
//      right after its own rounds (deeper links: one CTA-wide pass).
// Deliveries never leave the owning CTA, so the tick needs no scattered
// global atomics; the only global traffic is the owner blocks of the spiking
// rows, the spike list and the barrier.  The shared ring holds exactly the
// integers the global ring would, so results are bit-identical to the other
// launch shapes and to the oracle.
//
// The global ring stays the state of record between launches: a launch adds
// the global slot t%16 into tick t's arrivals during its first 16 ticks (and
// clears it), and at the end adds its shared window back into the global ring.
#include "net_device.cuh"

#include <stdexcept>

namespace ngb {
namespace {

using namespace netdev;

constexpr int RT = kResidentThreads;
constexpr int RW = RT / 32;
constexpr int kSlots = kOwnerBlockSlots;
constexpr unsigned long long kBarrierTimeoutNs = 2000000000ull; // 2 s
constexpr int kLinkCap = 512;  // queued overflow links per CTA-wide pass
constexpr int kWarpLinks = 32; // overflow links a warp queues for itself per tick

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_release_add_u32(unsigned *p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// 32-bit events (fp16 weights): bits 0-14 the weight's fp16 magnitude, 15-30
// the ring offset.  64-bit events (fp32 weights): bits 0-31 the fixed-point
// amount, 32-62 the ring offset.  The top bit marks a link word (index of the
// next block); all ones is an empty slot.
struct Ev32 {
  using word = uint32_t;
  static constexpr word kEmpty = 0xFFFFFFFFu;
  static constexpr word kLink = 0x80000000u;
  static constexpr int kDepth = 2; // rounds whose blocks are in flight beside the one delivered
  __device__ static uint32_t offset(word e) { return e >> 15; }
  __device__ static int amount(word e) { return quantum(half_bits(e & 0x7FFFu)); }
};

struct Ev64 {
  using word = unsigned long long;
  static constexpr word kEmpty = ~0ull;
  static constexpr word kLink = 1ull << 63;
  static constexpr int kDepth = 1;
  __device__ static uint32_t offset(word e) { return (uint32_t)(e >> 32); }
  __device__ static int amount(word e) { return (int)(uint32_t)e; }
};

// One owner block (8 words, 32-byte aligned) with 256-bit loads that take no
// L1 line: every lane of a warp reads a different row, so L1 would only cost
// tag work and line allocations for data that is used once.
__device__ __forceinline__ void ld_block256(const void *p, uint32_t (&v)[8]) {
  asm volatile("ld.global.L1::no_allocate.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
               : "l"(p));
}

template <class E> __device__ __forceinline__ void load_block(const typename E::word *p, typename E::word (&w)[kSlots]) {
  if constexpr (sizeof(typename E::word) == 4) {
    ld_block256(p, w);
  } else {
    uint32_t v[2][8];
    ld_block256(p, v[0]);
    ld_block256(reinterpret_cast<const uint32_t *>(p) + 8, v[1]);
#pragma unroll
    for (int k = 0; k < kSlots; ++k)
      w[k] = (unsigned long long)v[k >> 2][2 * (k & 3)] | ((unsigned long long)v[k >> 2][2 * (k & 3) + 1] << 32);
  }
}

// Ring position of an event at this tick: offset + 2P*(t mod Dr), wrapped
// once into [0, 2P*Dr) (offsets lie in [2P, 2P(Dr+1)), so one wrap suffices).
struct RingAt {
  int *ring; // shared ring as ints: [Dr][E, I][P]
  uint32_t tp2, lim2;
  template <class E> __device__ __forceinline__ void add(typename E::word e) const {
    const uint32_t u = E::offset(e) + tp2;
    atomicAdd(ring + min(u, u - lim2), E::amount(e));
  }
};

// Deliver one owner block and the overflow blocks it links to, by one lane;
// returns the number of events.  Empty slots only follow the filled ones.
// Links only point forward, so a chain ends; the hop bound only guards a
// corrupt table.
template <class E>
__device__ __forceinline__ int deliver_block(const RingAt &ra, const typename E::word *blocks,
                                             typename E::word (&w)[kSlots]) {
  int n = 0;
  for (int hop = 0; hop < (1 << 24); ++hop) {
#pragma unroll
    for (int j = 0; j < kSlots - 1; ++j) {
      if (w[j] == E::kEmpty) return n;
      ra.add<E>(w[j]);
      ++n;
    }
    const typename E::word last = w[kSlots - 1];
    if (last == E::kEmpty) return n;
    if (!(last & E::kLink)) {
      ra.add<E>(last);
      return n + 1;
    }
    load_block<E>(blocks + (size_t)(last & ~E::kLink) * kSlots, w);
  }
  return n;
}

// Overflow links met while delivering: queued for later rounds (the queue
// holds block indices; a full queue falls back to walking the chain in place).
struct LinkQueue {
  int *q;
  int *n;
  int cap;
};

// One owner block a lane: all 8 slots decoded and delivered unconditionally
// (predicated, no early exit), so a lane's 8 deliveries are independent of one
// another; an overflow link is queued.  Returns the lane's event count.
template <class E>
__device__ __forceinline__ int deliver_lane(const RingAt &ra, const typename E::word *blocks,
                                            const typename E::word (&w)[kSlots], const LinkQueue &links) {
  using W = typename E::word;
  int n = 0;
#pragma unroll
  for (int j = 0; j < kSlots; ++j) {
    const W e = w[j];
    // Empty slots (all ones) carry the link bit, so the last slot's test also skips them.
    const bool ok = j < kSlots - 1 ? e != E::kEmpty : !(e & E::kLink);
    const uint32_t u = E::offset(e) + ra.tp2;
    const int amount = E::amount(e);
    if (ok) {
      atomicAdd(ra.ring + min(u, u - ra.lim2), amount);
      ++n;
    }
  }
  const W last = w[kSlots - 1];
  if (last != E::kEmpty && (last & E::kLink)) {
    const int at = atomicAdd(links.n, 1);
    if (at < links.cap) {
      links.q[at] = (int)(last & ~E::kLink);
    } else {
      W b[kSlots];
      load_block<E>(blocks + (size_t)(last & ~E::kLink) * kSlots, b);
      n += deliver_block<E>(ra, blocks, b);
    }
  }
  return n;
}

// Grid-wide barrier over the co-resident CTAs of a cooperative launch, with a
// bounded wait: on a timeout (or another CTA's) the error flag is set and every
// CTA returns false.  Thread 0 also reads *count (complete once every CTA has
// arrived) into count_s.
__device__ __forceinline__ bool grid_sync(const ResidentDev &r, unsigned target, const unsigned *count, int &ok_s,
                                          int &count_s) {
  __syncthreads(); // the CTA's writes happen before thread 0's (cumulative) release
  if (threadIdx.x == 0) {
    red_release_add_u32(r.sync, 1u);
    int ok = 1;
    const unsigned long long start = global_ns();
    unsigned spin = 0;
    while (ld_acquire_u32(r.sync) < target) {
      if ((++spin & 63u) == 0u) {
        if (*(volatile int *)r.err) {
          ok = 0;
          break;
        }
        if (global_ns() - start > kBarrierTimeoutNs) {
          atomicExch(r.err, 1);
          ok = 0;
          break;
        }
      }
    }
    ok_s = ok;
    count_s = (int)__ldcg(count);
  }
  __syncthreads(); // thread 0's acquire happens before the CTA's later reads
  return ok_s != 0;
}

// Read and clear a neuron's (E, I) arrivals in its shared ring slot.
__device__ __forceinline__ int2 take_slot(int *slot, int P) {
  const int2 q = make_int2(slot[0], slot[P]);
  slot[0] = 0;
  slot[P] = 0;
  return q;
}

// Add a neuron's arrivals waiting in the global ring (the state of record
// between launches) and clear them.
__device__ __forceinline__ void take_global(int2 *g, int2 &q) {
  const int2 x = *g;
  if (x.x | x.y) {
    q.x += x.x;
    q.y += x.y;
    *g = make_int2(0, 0);
  }
}

__device__ __forceinline__ unsigned long long block_sum(unsigned long long v, unsigned long long *red_s) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
  __syncthreads();
  if (lane == 0) red_s[warp] = v;
  __syncthreads();
  unsigned long long s = 0;
  if (threadIdx.x == 0)
    for (int k = 0; k < RW; ++k) s += red_s[k];
  return s; // valid in thread 0
}

template <class E>
__global__ void __launch_bounds__(RT, 1) k_net_resident(NetDev d, ResidentDev r, long long t0, int ticks,
                                                        uint32_t *spikes_out, unsigned long long *counts, int words) {
  using W = typename E::word;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ unsigned long long red_s[RW];
  __shared__ int ok_s, spikes_s, link_n_s[2], warp_n_s[RW];
  const int C = r.ctas, P = r.per_cta, Dr = r.ring_depth, dr_mask = Dr - 1;
  const int c = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gbase = c * P;
  const int Pc = min(P, d.n - gbase);
  const int Pw = (Pc + 31) >> 5;
  int *ring_s = reinterpret_cast<int *>(smem); // [Dr][E, I][P]
  float *v_s = reinterpret_cast<float *>(ring_s + (size_t)Dr * 2 * P);
  float *a_s = v_s + P, *ge_s = a_s + P, *gi_s = ge_s + P;
  int *ref_s = reinterpret_cast<int *>(gi_s + P);
  uint32_t *word_s = reinterpret_cast<uint32_t *>(ref_s + P); // [P/32], P <= 2048
  int *link_q = reinterpret_cast<int *>(word_s + P / 32);      // [2][kLinkCap]
  int *warp_q = link_q + 2 * kLinkCap;                          // [RW][kWarpLinks]
  const W *blocks = static_cast<const W *>(r.blocks);

  for (int i = tid; i < Pc; i += RT) {
    v_s[i] = d.v[gbase + i];
    a_s[i] = d.a[gbase + i];
    ge_s[i] = d.ge[gbase + i];
    gi_s[i] = d.gi[gbase + i];
    ref_s[i] = d.ref[gbase + i];
  }
  for (int i = tid; i < Dr * 2 * P; i += RT) ring_s[i] = 0;
  if (tid == 0) link_n_s[0] = link_n_s[1] = 0;
  if (lane == 0) warp_n_s[warp] = 0;
  __syncthreads();

  unsigned long long events = 0, spikes = 0;
  for (int k = 0; k < ticks; ++k) {
    const long long t = t0 + k;
    const int par = (int)(t & 1), mod3 = (int)(t % 3);
    // 1. Membrane update of the held neurons.
    const int rs = (int)(t & dr_mask);
    const bool inflow = k < kRingSlots;
    if (Pc > RT) {
      // Two neurons a thread (P <= 2 * RT), computed side by side so their
      // dependent chains interleave; where the second does not exist, a
      // duplicate of neuron 0 is computed and discarded.
      const int i0 = tid, i1 = tid + RT;
      const bool ok0 = i0 < Pc, ok1 = i1 < Pc;
      const int j0 = ok0 ? i0 : 0, j1 = ok1 ? i1 : 0;
      int2 q0 = make_int2(0, 0), q1 = make_int2(0, 0);
      if (ok0) q0 = take_slot(ring_s + rs * 2 * P + j0, P);
      if (ok1) q1 = take_slot(ring_s + rs * 2 * P + j1, P);
      if (inflow) {
        int2 *g = d.ring + (size_t)(t & (kRingSlots - 1)) * d.n + gbase;
        if (ok0) take_global(g + j0, q0);
        if (ok1) take_global(g + j1, q1);
      }
      float v0 = v_s[j0], a0 = a_s[j0], e0 = ge_s[j0], n0 = gi_s[j0];
      float v1 = v_s[j1], a1 = a_s[j1], e1 = ge_s[j1], n1 = gi_s[j1];
      int r0 = ref_s[j0], r1 = ref_s[j1];
      const bool s0 = alif_math(d, t, gbase + j0, q0, v0, a0, e0, n0, r0) && ok0;
      const bool s1 = alif_math(d, t, gbase + j1, q1, v1, a1, e1, n1, r1) && ok1;
      if (ok0) {
        v_s[j0] = v0;
        a_s[j0] = a0;
        ge_s[j0] = e0;
        gi_s[j0] = n0;
        ref_s[j0] = r0;
      }
      if (ok1) {
        v_s[j1] = v1;
        a_s[j1] = a1;
        ge_s[j1] = e1;
        gi_s[j1] = n1;
        ref_s[j1] = r1;
      }
      const unsigned f0 = __ballot_sync(0xffffffffu, s0);
      const unsigned f1 = __ballot_sync(0xffffffffu, s1);
      if (lane == 0) {
        if ((i0 >> 5) < Pw) word_s[i0 >> 5] = f0;
        if ((i1 >> 5) < Pw) word_s[i1 >> 5] = f1;
      }
    } else {
      // One neuron a thread (small networks).
      bool s0 = false;
      if (tid < Pc) {
        int2 q = take_slot(ring_s + rs * 2 * P + tid, P);
        if (inflow) take_global(d.ring + (size_t)(t & (kRingSlots - 1)) * d.n + gbase + tid, q);
        s0 = alif_math(d, t, gbase + tid, q, v_s[tid], a_s[tid], ge_s[tid], gi_s[tid], ref_s[tid]);
      }
      const unsigned f0 = __ballot_sync(0xffffffffu, s0);
      if (lane == 0 && (tid >> 5) < Pw) word_s[tid >> 5] = f0;
    }
    __syncthreads();
    // 2. This CTA's spike ids into its reserved range of the tick's list.
    if (warp == 0) {
      const uint32_t w0 = lane < Pw ? word_s[lane] : 0u;
      const uint32_t w1 = lane + 32 < Pw ? word_s[lane + 32] : 0u;
      const int own = __popc(w0) + __popc(w1);
      int incl = own;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      const int total = __shfl_sync(0xffffffffu, incl, 31);
      int base = 0;
      if (lane == 0 && total) base = (int)atomicAdd(r.sync + 1 + mod3, (unsigned)total);
      base = __shfl_sync(0xffffffffu, base, 0);
      int *lst = r.lists + (size_t)par * d.n_pre;
      int at = base + incl - own;
      for (uint32_t m = w0; m; m &= m - 1) lst[at++] = gbase + lane * 32 + (__ffs(m) - 1);
      for (uint32_t m = w1; m; m &= m - 1) lst[at++] = gbase + (lane + 32) * 32 + (__ffs(m) - 1);
      if (spikes_out) {
        uint32_t *row = spikes_out + (size_t)k * words + (gbase >> 5);
        if (lane < Pw) row[lane] = w0;
        if (lane + 32 < Pw) row[lane + 32] = w1;
      }
      if (lane == 0) {
        spikes += (unsigned long long)total;
        if (counts && total) atomicAdd(counts + 2 * (size_t)k, (unsigned long long)total);
      }
    }
    // 3. Past the barrier every CTA's ids are in the list, and spikes_s holds their number.
    if (!grid_sync(r, (unsigned)C * (unsigned)(k + 1) + (unsigned)r.stall_test, r.sync + 1 + mod3, ok_s, spikes_s))
      return;
    // Tick t-1's counter has been read by every CTA: clear it for tick t+2.
    if (c == 0 && tid == 0) r.sync[1 + (int)((t + 2) % 3)] = 0u;
    // 4. Deliver the owner blocks (p, c) of this tick's spikes.
    const int S = spikes_s, R = (S + 31) >> 5;
    const int *lst = r.lists + (size_t)par * d.n_pre;
    const RingAt ra{ring_s, (uint32_t)(2 * P * (int)(t & dr_mask)), (uint32_t)(2 * P * Dr)};
    const LinkQueue links0{link_q, &link_n_s[0], kLinkCap};
    const LinkQueue own_links{warp_q + warp * kWarpLinks, &warp_n_s[warp], kWarpLinks};
    constexpr int D = E::kDepth;
    // This warp's rounds are warp + m*RW, m < M; the blocks of rounds m+1..m+D
    // are in flight while round m is delivered (buffers renamed statically).
    const int M = R > warp ? (R - warp + RW - 1) / RW : 0;
    auto list_at = [&](int m) -> int {
      const int i = (warp + m * RW) * 32 + lane;
      return (m < M && i < S) ? __ldcg(lst + i) : -1;
    };
    auto fetch = [&](int p, W (&w)[kSlots]) {
      if (p >= 0) {
        load_block<E>(blocks + ((size_t)p * C + c) * kSlots, w);
      } else {
#pragma unroll
        for (int j = 0; j < kSlots; ++j) w[j] = E::kEmpty;
      }
    };
    unsigned long long tick_events = 0;
    W b[D + 1][kSlots];
    {
      int p0[D];
#pragma unroll
      for (int j = 0; j < D; ++j) p0[j] = list_at(j);
#pragma unroll
      for (int j = 0; j < D; ++j) fetch(p0[j], b[j]);
    }
    int pn = list_at(D);
    for (int m = 0; m < M; m += D + 1) {
#pragma unroll
      for (int ph = 0; ph <= D; ++ph) {
        if (m + ph < M) {
          fetch(pn, b[(ph + D) % (D + 1)]); // round m + ph + D
          pn = list_at(m + ph + D + 1);
          tick_events += (unsigned long long)deliver_lane<E>(ra, blocks, b[ph], own_links);
        }
      }
    }
    // The overflow blocks this warp met, delivered by the warp itself while the
    // others may still be in their rounds; their own links go to the CTA queue.
    __syncwarp();
    {
      const int n = min(warp_n_s[warp], kWarpLinks);
      if (n > 0) {
        W w[kSlots];
        if (lane < n) {
          load_block<E>(blocks + (size_t)own_links.q[lane] * kSlots, w);
        } else {
#pragma unroll
          for (int j = 0; j < kSlots; ++j) w[j] = E::kEmpty;
        }
        tick_events += (unsigned long long)deliver_lane<E>(ra, blocks, w, links0);
      }
      __syncwarp();
      if (lane == 0) warp_n_s[warp] = 0;
    }
    __syncthreads();
    // Overflow blocks, in rounds of 32; their own links go to the other queue.
    for (int pass = 0; pass < 64; ++pass) {
      const int cur = pass & 1;
      const int n = min(link_n_s[cur], kLinkCap);
      if (n == 0) break;
      const int *q = link_q + cur * kLinkCap;
      const LinkQueue next{link_q + (cur ^ 1) * kLinkCap, &link_n_s[cur ^ 1], kLinkCap};
      for (int rr = warp; rr * 32 < n; rr += RW) {
        const int i = rr * 32 + lane;
        W w[kSlots];
        if (i < n) {
          load_block<E>(blocks + (size_t)q[i] * kSlots, w);
        } else {
#pragma unroll
          for (int j = 0; j < kSlots; ++j) w[j] = E::kEmpty;
        }
        tick_events += (unsigned long long)deliver_lane<E>(ra, blocks, w, next);
      }
      __syncthreads();
      if (tid == 0) link_n_s[cur] = 0;
      __syncthreads();
    }
    events += tick_events;
    if (counts) {
      const unsigned long long s = block_sum(tick_events, red_s);
      if (tid == 0 && s) atomicAdd(counts + 2 * (size_t)k + 1, s);
    }
  }

  // Write the state back; add the shared ring window [t_end, t_end + Dr) into
  // the global ring.
  __syncthreads();
  const long long te = t0 + ticks;
  for (int i = tid; i < Pc; i += RT) {
    d.v[gbase + i] = v_s[i];
    d.a[gbase + i] = a_s[i];
    d.ge[gbase + i] = ge_s[i];
    d.gi[gbase + i] = gi_s[i];
    d.ref[gbase + i] = ref_s[i];
    for (int j = 0; j < Dr; ++j) {
      const long long tt = te + j;
      const int *slot = ring_s + (int)(tt & dr_mask) * 2 * P + i;
      const int2 q = make_int2(slot[0], slot[P]);
      if (q.x | q.y) {
        int2 *g = d.ring + (size_t)(tt & (kRingSlots - 1)) * d.n + gbase + i;
        int2 x = *g;
        x.x += q.x;
        x.y += q.y;
        *g = x;
      }
    }
  }
  const unsigned long long ev = block_sum(events, red_s);
  if (tid == 0) {
    d.totals[kTotalsStride * (size_t)c] += spikes;
    d.totals[kTotalsStride * (size_t)c + 1] += ev;
  }
}

// ---- owner-block construction (once per network) ----

__device__ __forceinline__ int chain_blocks(int n) {
  if (n <= kSlots) return 0;
  const int rem = n - (kSlots - 1);
  const int m = (rem - 1 + kSlots - 2) / (kSlots - 1);
  return m > 1 ? m : 1;
}

template <bool HALF> __device__ __forceinline__ uint32_t weight_bits(const NetDev &d, long long e) {
  if (HALF) return static_cast<const uint16_t *>(d.w)[e];
  return __float_as_uint(static_cast<const float *>(d.w)[e]);
}

template <bool HALF> __device__ __forceinline__ float weight_of(uint32_t bits) {
  return HALF ? half_bits(bits) : __uint_as_float(bits);
}

// Event word: ring offset 2*d*P + (P if w < 0) + post with the fp16 magnitude
// (32-bit events) or the fixed-point amount (64-bit events).
template <class E> __device__ __forceinline__ typename E::word encode(uint32_t wbits, float w, uint32_t off);
template <> __device__ __forceinline__ uint32_t encode<Ev32>(uint32_t wbits, float, uint32_t off) {
  return (wbits & 0x7FFFu) | (off << 15);
}
template <> __device__ __forceinline__ unsigned long long encode<Ev64>(uint32_t, float w, uint32_t off) {
  return (unsigned long long)(uint32_t)quantum(w) | ((unsigned long long)off << 32);
}

template <bool HALF> __device__ __forceinline__ bool is_zero(uint32_t bits) {
  return HALF ? (bits & 0x7FFFu) == 0u : (bits & 0x7FFFFFFFu) == 0u;
}

constexpr int BT = 256;

// Synapses of presynaptic neuron `pre`, by index e.  CSR: entries
// [row[pre], row[pre+1]).  Block storage: e = block * 16 + r over the blocks of
// the pre's block-column, i.e. entry r of the pre's column in each 16x16 tile
// (zero entries are skipped by the callers, as they are by the block push).
template <bool BSR> __device__ __forceinline__ void edge_range(const NetDev &d, int pre, long long &e0, long long &e1) {
  if (BSR) {
    e0 = d.bcol[pre >> 4] * 16;
    e1 = d.bcol[(pre >> 4) + 1] * 16;
  } else {
    e0 = d.row[pre];
    e1 = d.row[pre + 1];
  }
}
// The synapse word post | (delay - 1) << 28 of entry e.
template <bool BSR> __device__ __forceinline__ uint32_t edge_word(const NetDev &d, long long e) {
  if (BSR) {
    const uint32_t m = d.blk[e >> 4];
    return ((m & kPostMask) * 16u + (uint32_t)(e & 15)) | (m & ~kPostMask);
  }
  return d.syn[e];
}
template <bool BSR, bool HALF> __device__ __forceinline__ uint32_t edge_weight(const NetDev &d, int pre, long long e) {
  if (BSR) return d.tiles[((size_t)(e >> 4) * 16 + (pre & 15)) * 16 + (e & 15)];
  return weight_bits<HALF>(d, e);
}

// CTA per presynaptic row: non-zero synapses per owner CTA -> overflow blocks needed.
template <bool BSR, bool HALF> __global__ void __launch_bounds__(BT) k_owner_count(NetDev d, ResidentDev r,
                                                                                  unsigned long long *need) {
  extern __shared__ int cnt[];
  __shared__ unsigned long long red_s[BT / 32];
  const int pre = blockIdx.x, C = r.ctas, P = r.per_cta;
  for (int q = threadIdx.x; q < C; q += BT) cnt[q] = 0;
  __syncthreads();
  long long e0, e1;
  edge_range<BSR>(d, pre, e0, e1);
  for (long long e = e0 + threadIdx.x; e < e1; e += BT)
    if (!is_zero<HALF>(edge_weight<BSR, HALF>(d, pre, e)))
      atomicAdd(&cnt[(int)(edge_word<BSR>(d, e) & kPostMask) / P], 1);
  __syncthreads();
  unsigned long long extra = 0;
  for (int q = threadIdx.x; q < C; q += BT) extra += (unsigned long long)chain_blocks(cnt[q]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) extra += __shfl_down_sync(0xffffffffu, extra, o);
  if ((threadIdx.x & 31) == 0) red_s[threadIdx.x >> 5] = extra;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long s = 0;
    for (int k = 0; k < BT / 32; ++k) s += red_s[k];
    if (s) atomicAdd(need, s);
  }
}

// CTA per presynaptic row: writes its owner blocks (pre-filled with empty
// words) and allocates overflow blocks from `cursor`.
template <class E, bool BSR, bool HALF>
__global__ void __launch_bounds__(BT) k_owner_fill(NetDev d, ResidentDev r, typename E::word *blocks,
                                                   unsigned long long *cursor, unsigned long long capacity,
                                                   int *err) {
  extern __shared__ long long fill_s[];
  const int pre = blockIdx.x, C = r.ctas, P = r.per_cta;
  long long *chain = fill_s;                               // [C]
  int *cnt = reinterpret_cast<int *>(fill_s + C);          // [C]
  int *cur = cnt + C;                                      // [C]
  const unsigned long long primary = (unsigned long long)d.n_pre * C;
  for (int q = threadIdx.x; q < C; q += BT) cnt[q] = cur[q] = 0;
  __syncthreads();
  long long e0, e1;
  edge_range<BSR>(d, pre, e0, e1);
  for (long long e = e0 + threadIdx.x; e < e1; e += BT)
    if (!is_zero<HALF>(edge_weight<BSR, HALF>(d, pre, e)))
      atomicAdd(&cnt[(int)(edge_word<BSR>(d, e) & kPostMask) / P], 1);
  __syncthreads();
  for (int q = threadIdx.x; q < C; q += BT) {
    const int m = chain_blocks(cnt[q]);
    long long base = -1;
    if (m) {
      const unsigned long long b = atomicAdd(cursor, (unsigned long long)m);
      if (b + m <= capacity) base = (long long)(primary + b);
      else atomicExch(err, 2);
    }
    chain[q] = base;
  }
  __syncthreads();
  for (long long e = e0 + threadIdx.x; e < e1; e += BT) {
    const uint32_t wb = edge_weight<BSR, HALF>(d, pre, e);
    if (is_zero<HALF>(wb)) continue;
    const uint32_t word = edge_word<BSR>(d, e);
    const int post = (int)(word & kPostMask), q = post / P;
    const int s = atomicAdd(&cur[q], 1), n = cnt[q];
    long long blk = (long long)pre * C + q;
    int j = s;
    if (n > kSlots && s >= kSlots - 1) {
      if (chain[q] < 0) continue;
      const int m = chain_blocks(n), s2 = s - (kSlots - 1);
      const int kq = min(s2 / (kSlots - 1), m - 1);
      j = s2 - kq * (kSlots - 1);
      blk = chain[q] + kq;
    }
    const uint32_t off = 2u * (uint32_t)(((int)(word >> 28) + 1) * P) + (weight_of<HALF>(wb) < 0.f ? (uint32_t)P : 0u) +
                         (uint32_t)(post - q * P);
    blocks[(size_t)blk * kSlots + j] = encode<E>(wb, weight_of<HALF>(wb), off);
  }
  for (int q = threadIdx.x; q < C; q += BT) {
    const int n = cnt[q];
    if (n <= kSlots || chain[q] < 0) continue;
    const int m = chain_blocks(n);
    blocks[((size_t)pre * C + q) * kSlots + kSlots - 1] = E::kLink | (typename E::word)chain[q];
    for (int kq = 0; kq + 1 < m; ++kq)
      blocks[(size_t)(chain[q] + kq) * kSlots + kSlots - 1] = E::kLink | (typename E::word)(chain[q] + kq + 1);
  }
}

template <class E> void *resident_kernel() { return reinterpret_cast<void *>(&k_net_resident<E>); }

} // namespace

size_t resident_smem_bytes(const ResidentDev &r) {
  const size_t P = size_t(r.per_cta);
  return size_t(r.ring_depth) * P * 8 + P * 20 + (P / 32) * 4 + 2 * size_t(kLinkCap) * 4 +
         size_t(RW) * kWarpLinks * 4;
}

int resident_max_ctas(bool ev64, size_t smem) {
  void *fn = ev64 ? resident_kernel<Ev64>() : resident_kernel<Ev32>();
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess) {
    (void)cudaGetLastError();
    return 0;
  }
  int per_sm = 0, dev = 0, sms = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, RT, smem) != cudaSuccess) {
    (void)cudaGetLastError();
    return 0;
  }
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return per_sm * sms;
}

cudaError_t launch_net_resident(const NetDev &d, const ResidentDev &r, long long t0, int ticks, uint32_t *spikes_out,
                                unsigned long long *counts, int words, cudaStream_t s) {
  NetDev dd = d;
  ResidentDev rr = r;
  void *args[] = {&dd, &rr, &t0, &ticks, &spikes_out, &counts, &words};
  void *fn = r.ev64 ? resident_kernel<Ev64>() : resident_kernel<Ev32>();
  const size_t smem = resident_smem_bytes(r);
  const cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  return cudaLaunchCooperativeKernel(fn, dim3(r.ctas), dim3(RT), args, smem, s);
}

void launch_owner_count(const NetDev &d, const ResidentDev &r, unsigned long long *need, cudaStream_t s) {
  if (d.n_pre == 0) return;
  const size_t smem = size_t(r.ctas) * 4;
  if (d.bsr) k_owner_count<true, true><<<d.n_pre, BT, smem, s>>>(d, r, need);
  else if (d.w_half) k_owner_count<false, true><<<d.n_pre, BT, smem, s>>>(d, r, need);
  else k_owner_count<false, false><<<d.n_pre, BT, smem, s>>>(d, r, need);
}

void launch_owner_fill(const NetDev &d, const ResidentDev &r, void *blocks, unsigned long long *cursor,
                       unsigned long long capacity, int *err, cudaStream_t s) {
  if (d.n_pre == 0) return;
  const size_t smem = size_t(r.ctas) * 16;
  if (d.bsr) {
    // Block storage holds fp16 weights: 32-bit events.
    if (r.ev64) throw std::logic_error("block storage takes 32-bit owner events");
    k_owner_fill<Ev32, true, true><<<d.n_pre, BT, smem, s>>>(d, r, static_cast<uint32_t *>(blocks), cursor, capacity,
                                                              err);
  } else if (r.ev64) {
    k_owner_fill<Ev64, false, false><<<d.n_pre, BT, smem, s>>>(d, r, static_cast<unsigned long long *>(blocks),
                                                                cursor, capacity, err);
  } else {
    if (!d.w_half) throw std::logic_error("32-bit owner events need fp16 weights");
    k_owner_fill<Ev32, false, true><<<d.n_pre, BT, smem, s>>>(d, r, static_cast<uint32_t *>(blocks), cursor,
                                                               capacity, err);
  }
}

} // namespace ngb
