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
// another; an overflow link is queued, in `spill` when `links` is full (a
// chain walked in place would hold up the lane's whole warp for a dependent
// read).  Returns the lane's event count.
template <class E>
__device__ __forceinline__ int deliver_lane(const RingAt &ra, const typename E::word *blocks,
                                            const typename E::word (&w)[kSlots], const LinkQueue &links,
                                            const LinkQueue *spill = nullptr) {
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
    const int link = (int)(last & ~E::kLink);
    const int at = atomicAdd(links.n, 1);
    if (at < links.cap) {
      links.q[at] = link;
      return n;
    }
    if (spill) {
      const int at2 = atomicAdd(spill->n, 1);
      if (at2 < spill->cap) {
        spill->q[at2] = link;
        return n;
      }
    }
    W b[kSlots];
    load_block<E>(blocks + (size_t)link * kSlots, b);
    n += deliver_block<E>(ra, blocks, b);
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
          tick_events += (unsigned long long)deliver_lane<E>(ra, blocks, b[ph], own_links, &links0);
        }
      }
    }
    // The overflow blocks this warp met, delivered by the warp itself while the
    // others may still be in their rounds; their own links, and those its full
    // queue spilled, go to the CTA queue.
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

// ---- pipelined tick ----
//
// The serial tick above keeps the membrane update, the spike list and the
// grid barrier on the critical path ahead of each delivery.  The pipelined
// tick splits the CTA into two warp groups:
//
//   membrane group (MW warps): tick t's membrane update; the tick's spike
//     list (warp 0); the delay-1 synapses of the CTA's spiking neurons, pushed
//     straight into the global ring slot of tick t+1 with global atomics
//     (warps 1..MW-1; about 1/8 of the events at delays 1-8, read as
//     contiguous row segments); arrival at the grid barrier, whose completion
//     thread 0 waits for and announces to the CTA.
//   delivery group (the other warps): the owner blocks of tick t's spikes,
//     which hold only delay>=2 synapses here, into the shared ring, while the
//     membrane group already runs tick t+1.
//
// Dependencies of tick t: its membrane update needs the barrier of tick t-1
// (every CTA's delay-1 pushes are in the global slot t) and the delivery of
// tick t-2 (the last one that adds into the shared slot t); the delivery of
// tick t needs the barrier of tick t (the list is complete).  The groups hand
// over through shared-memory mbarriers, four of each kind indexed by k % 4, so
// that a phase parity cannot alias (the groups are never more than two ticks
// apart).  Lists rotate over three buffers by t % 3: a CTA still delivering
// tick t-1 has already arrived at the barrier of tick t, so another CTA can be
// writing the list of tick t+1, but not of tick t+2.
// Everything a delivery adds is an integer, so the sums, and the results, are
// bit-identical to the serial tick, the other launch shapes and the oracle.

constexpr unsigned long long kGroupWaitNs = 4000000000ull; // 4 s, above the grid barrier's 2 s

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mb_init(unsigned long long *mb, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(mb)), "r"(count) : "memory");
}

// Arrive (release at CTA scope: this thread's earlier writes, and those it has
// observed through a barrier, happen before the waiters' later reads).
__device__ __forceinline__ void mb_arrive(unsigned long long *mb) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(mb)) : "memory");
}

__device__ __forceinline__ bool mb_test(unsigned long long *mb, unsigned parity) {
  uint32_t ok;
  asm volatile("{\n\t.reg .pred p;\n\t"
               "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
               "selp.u32 %0, 1, 0, p;\n\t}"
               : "=r"(ok)
               : "r"(smem_u32(mb)), "r"(parity)
               : "memory");
  return ok != 0;
}

// Bounded wait for the completion of the phase with this parity; false when
// it did not complete within kGroupWaitNs.
__device__ __forceinline__ bool mb_wait(unsigned long long *mb, unsigned parity) {
  if (mb_test(mb, parity)) return true;
  const unsigned long long start = global_ns();
  for (unsigned spin = 1; spin < (1u << 30); ++spin) {
    if (mb_test(mb, parity)) return true;
    if ((spin & 15u) == 0u && global_ns() - start > kGroupWaitNs) return false;
  }
  return false;
}

// Named barrier of one warp group (id 1: membrane, 2: delivery).
__device__ __forceinline__ void group_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// Named barrier that also returns whether any thread of the group passed true
// (a decision every thread of the group takes alike).
__device__ __forceinline__ bool group_any(int id, int n, bool v) {
  uint32_t res;
  asm volatile("{\n\t.reg .pred p, q;\n\t"
               "setp.ne.u32 p, %1, 0;\n\t"
               "bar.red.or.pred q, %2, %3, p;\n\t"
               "selp.u32 %0, 1, 0, q;\n\t}"
               : "=r"(res)
               : "r"((uint32_t)v), "r"(id), "r"(n)
               : "memory");
  return res != 0;
}

// Add a delay-1 synapse of weight w onto post in the global slot gslot
// (int pairs E, I); returns 1 if it carried an event.
__device__ __forceinline__ int push_event(int *gslot, uint32_t word, float w) {
  if (w == 0.f) return 0;
  atomicAdd(gslot + 2 * (size_t)(word & kPostMask) + (w < 0.f ? 1 : 0), quantum(w));
  return 1;
}

// Delay-1 segment of a CSR row, entries [e0, e0 + len) (len and e0 multiples
// of 8): lane chunk ch (0..7) takes entries ch*8 .. ch*8+7 of each 64-entry
// pass, one 32-byte index load and one 16- or 32-byte weight load.
template <bool HALF>
__device__ __forceinline__ int push_d1_row(const NetDev &d, int *gslot, long long e0, int len, int ch, int passes) {
  int n = 0;
  for (int ps = 0; ps < passes; ++ps) {
    const int off = ps * 64 + ch * 8;
    if (off >= len) continue;
    const long long e = e0 + off;
    const uint4 *sp = reinterpret_cast<const uint4 *>(d.syn + e);
    const uint4 s0 = __ldcs(sp), s1 = __ldcs(sp + 1);
    float w[8];
    if (HALF) {
      const uint4 wv = __ldcs(reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(d.w) + e));
      const uint32_t h[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        w[2 * j] = half_bits(h[j] & 0xFFFFu);
        w[2 * j + 1] = half_bits(h[j] >> 16);
      }
    } else {
      const float4 *wp = reinterpret_cast<const float4 *>(static_cast<const float *>(d.w) + e);
      const float4 f0 = __ldcs(wp), f1 = __ldcs(wp + 1);
      w[0] = f0.x; w[1] = f0.y; w[2] = f0.z; w[3] = f0.w;
      w[4] = f1.x; w[5] = f1.y; w[6] = f1.z; w[7] = f1.w;
    }
    const uint32_t word[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) n += push_event(gslot, word[j], w[j]);
  }
  return n;
}

// Delay-1 blocks [b0, b0 + nb) of a block-column, column `col` of each tile
// (16 fp16 weights, one 32-byte sector): lane chunk ch takes blocks ch, ch+8, ...
__device__ __forceinline__ int push_d1_blocks(const NetDev &d, int *gslot, int col, long long b0, int nb, int ch) {
  int n = 0;
  for (int b = ch; b < nb; b += 8) {
    const long long bb = b0 + b;
    const uint32_t meta = __ldcs(d.blk + bb);
    const uint4 *cp = reinterpret_cast<const uint4 *>(d.tiles + ((size_t)bb * 16 + col) * 16);
    const uint4 c0 = __ldcs(cp), c1 = __ldcs(cp + 1);
    const uint32_t post0 = (meta & kPostMask) * 16u;
    const uint32_t h[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      n += push_event(gslot, post0 + 2 * j, half_bits(h[j] & 0xFFFFu));
      n += push_event(gslot, post0 + 2 * j + 1, half_bits(h[j] >> 16));
    }
  }
  return n;
}

template <class E, bool BSR, int MW>
__global__ void __launch_bounds__(RT, 1) k_net_pipe(NetDev d, ResidentDev r, long long t0, int ticks,
                                                    uint32_t *spikes_out, unsigned long long *counts, int words) {
  using W = typename E::word;
  constexpr int MT = MW * 32, DW = RW - MW, DT = DW * 32;
  constexpr int JN = (2048 + MT - 1) / MT; // neurons a membrane thread holds (P <= 2048)
  constexpr int PW = MW - 1;               // pushing warps: 1..MW-1 (warp 0 writes the list)
  constexpr int NI = (64 + PW - 1) / PW;   // spike words a pushing warp covers (at most 64 a CTA)
  constexpr unsigned FULL = 0xffffffffu;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ unsigned long long red_s[RW];
  __shared__ unsigned long long mb_grid[4], mb_done[4];
  __shared__ int cnt_s[4], abort_s, link_n_s[2], warp_n_s[RW];
  const int C = r.ctas, P = r.per_cta, Dr = r.ring_depth, dr_mask = Dr - 1;
  const int c = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gbase = c * P;
  const int Pc = min(P, d.n - gbase);
  const int Pw = (Pc + 31) >> 5;
  int *ring_s = reinterpret_cast<int *>(smem); // [Dr][E, I][P]
  float *v_s = reinterpret_cast<float *>(ring_s + (size_t)Dr * 2 * P);
  float *a_s = v_s + P, *ge_s = a_s + P, *gi_s = ge_s + P;
  int *ref_s = reinterpret_cast<int *>(gi_s + P);
  uint32_t *word_s = reinterpret_cast<uint32_t *>(ref_s + P); // [P/32]
  int *link_q = reinterpret_cast<int *>(word_s + P / 32);      // [2][kLinkCap]
  int *warp_q = link_q + 2 * kLinkCap;                          // [RW][kWarpLinks]
  // Delay-1 segments of the held neurons: CSR (row offset from the CTA's first
  // row, length) per neuron; block storage (first block, count) per block-column.
  const size_t meta_at = ((size_t)(reinterpret_cast<unsigned char *>(warp_q + RW * kWarpLinks) - smem) + 7) & ~size_t(7);
  uint2 *d1_s = reinterpret_cast<uint2 *>(smem + meta_at); // [P]
  long long *d1b_s = reinterpret_cast<long long *>(d1_s);   // [P/16]
  int *d1bn_s = reinterpret_cast<int *>(d1b_s + P / 16);     // [P/16]
  const W *blocks = static_cast<const W *>(r.blocks);

  for (int i = tid; i < Pc; i += RT) {
    v_s[i] = d.v[gbase + i];
    a_s[i] = d.a[gbase + i];
    ge_s[i] = d.ge[gbase + i];
    gi_s[i] = d.gi[gbase + i];
    ref_s[i] = d.ref[gbase + i];
  }
  for (int i = tid; i < Dr * 2 * P; i += RT) ring_s[i] = 0;
  long long row_base = 0;
  if (BSR) {
    for (int j = tid; j < (Pc + 15) >> 4; j += RT) {
      const int bc = (gbase >> 4) + j;
      d1b_s[j] = d.bcol[bc];
      d1bn_s[j] = d.bmid[bc];
    }
  } else {
    row_base = d.row[gbase];
    for (int i = tid; i < Pc; i += RT)
      d1_s[i] = make_uint2((uint32_t)(d.row[gbase + i] - row_base), (uint32_t)d.mid[gbase + i]);
  }
  if (tid == 0) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      mb_init(&mb_grid[j], 1);
      mb_init(&mb_done[j], DW);
      cnt_s[j] = 0;
    }
    abort_s = 0;
    link_n_s[0] = link_n_s[1] = 0;
  }
  if (lane == 0) warp_n_s[warp] = 0;
  __syncthreads();

  unsigned long long events = 0, spikes = 0;
  if (warp < MW) {
    // ---------------- membrane group ----------------
    for (int k = 0; k < ticks; ++k) {
      const long long t = t0 + k;
      bool bad = false;
      if (k >= 1) bad = !mb_wait(&mb_grid[(k - 1) & 3], ((k - 1) >> 2) & 1);
      if (k >= 2 && !bad) bad = !mb_wait(&mb_done[(k - 2) & 3], ((k - 2) >> 2) & 1);
      // abort_s is written before the arrival waited for, so every thread reads
      // the same value; the reduction makes a timeout's decision common too.
      if (group_any(1, MT, bad || abort_s != 0)) {
        if (tid == 0) {
          if (bad) atomicExch(r.err, 1);
          abort_s = 1;
          mb_arrive(&mb_grid[k & 3]); // release a delivery group waiting for tick t
        }
        break;
      }
      const int m3 = (int)(t % 3);
      const int rs = (int)(t & dr_mask);
      int2 *gslot = d.ring + (size_t)(t & (kRingSlots - 1)) * d.n + gbase;
      // 1. Membrane update.  The global slot's entries of all of the thread's
      //    neurons are read (at L2: other CTAs' atomics wrote them) and cleared
      //    first, one round trip, then the neurons are updated two at a time,
      //    their chains interleaved.
      int2 gq[JN];
#pragma unroll
      for (int j = 0; j < JN; ++j) {
        const int i = j * MT + tid;
        gq[j] = i < Pc ? __ldcg(gslot + i) : make_int2(0, 0);
      }
#pragma unroll
      for (int j = 0; j < JN; ++j) {
        const int i = j * MT + tid;
        if (i < Pc && (gq[j].x | gq[j].y)) __stcg(gslot + i, make_int2(0, 0));
      }
#pragma unroll
      for (int j = 0; j < JN; j += 2) {
        if (j * MT >= Pc) break;
        const int i0 = j * MT + tid, i1 = (j + 1) * MT + tid;
        const bool ok0 = i0 < Pc, ok1 = j + 1 < JN && i1 < Pc;
        const int j0 = ok0 ? i0 : 0, j1 = ok1 ? i1 : 0;
        const int2 g1 = gq[j + 1 < JN ? j + 1 : j];
        int2 q0 = make_int2(0, 0), q1 = make_int2(0, 0);
        if (ok0) {
          q0 = take_slot(ring_s + rs * 2 * P + j0, P);
          q0.x += gq[j].x;
          q0.y += gq[j].y;
        }
        if (ok1) {
          q1 = take_slot(ring_s + rs * 2 * P + j1, P);
          q1.x += g1.x;
          q1.y += g1.y;
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
        const unsigned f0 = __ballot_sync(FULL, s0);
        const unsigned f1 = __ballot_sync(FULL, s1);
        if (lane == 0) {
          if ((i0 >> 5) < Pw) word_s[i0 >> 5] = f0;
          if (j + 1 < JN && (i1 >> 5) < Pw) word_s[i1 >> 5] = f1;
        }
      }
      group_sync(1, MT);
      unsigned long long tick_events = 0;
      if (warp == 0) {
        // 2. The CTA's spike ids into its reserved range of the tick's list.
        const uint32_t w0 = lane < Pw ? word_s[lane] : 0u;
        const uint32_t w1 = lane + 32 < Pw ? word_s[lane + 32] : 0u;
        const int own = __popc(w0) + __popc(w1);
        int incl = own;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int v = __shfl_up_sync(FULL, incl, o);
          if (lane >= o) incl += v;
        }
        const int total = __shfl_sync(FULL, incl, 31);
        int base = 0;
        if (lane == 0 && total) base = (int)atomicAdd(r.sync + 1 + m3, (unsigned)total);
        base = __shfl_sync(FULL, base, 0);
        int *lst = r.lists + (size_t)m3 * d.n_pre;
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
      } else {
        // 3. Delay-1 synapses of the CTA's spiking neurons into the global
        //    slot of tick t+1: warp w takes words w-1, w-1+PW, ...; a group of
        //    8 lanes takes one spiking neuron at a time, four neurons a round.
        const int pw = warp - 1;
        int *gnext = reinterpret_cast<int *>(d.ring + (size_t)((t + 1) & (kRingSlots - 1)) * d.n);
        const int qi = pw + lane * PW;
        const uint32_t wq = (lane < NI && qi < Pw) ? word_s[qi] : 0u;
        const int cq = __popc(wq);
        int incl = cq;
#pragma unroll
        for (int o = 1; o < NI; o <<= 1) {
          const int v = __shfl_up_sync(FULL, incl, o);
          if (lane >= o) incl += v;
        }
        const int total = __shfl_sync(FULL, incl, NI - 1);
        const int grp = lane >> 3, ch = lane & 7;
        for (int r0 = 0; r0 < total; r0 += 4) {
          const int rk = r0 + grp;
          int li = -1;
#pragma unroll
          for (int i = 0; i < NI; ++i) {
            const int inc = __shfl_sync(FULL, incl, i), cnt = __shfl_sync(FULL, cq, i);
            const uint32_t wi = __shfl_sync(FULL, wq, i);
            if (li < 0 && rk < total && rk < inc) {
              uint32_t m = wi;
              for (int s = rk - (inc - cnt); s > 0; --s) m &= m - 1;
              li = (pw + i * PW) * 32 + (__ffs(m) - 1);
            }
          }
          if (BSR) {
            const long long b0 = li >= 0 ? d1b_s[li >> 4] : 0;
            const int nb = li >= 0 ? d1bn_s[li >> 4] : 0;
            tick_events += (unsigned long long)push_d1_blocks(d, gnext, (gbase + max(li, 0)) & 15, b0, nb, ch);
          } else {
            const uint2 m = li >= 0 ? d1_s[li] : make_uint2(0u, 0u);
            const int passes = (int)((__reduce_max_sync(FULL, m.y) + 63u) >> 6);
            tick_events += (unsigned long long)push_d1_row<sizeof(W) == 4>(d, gnext, row_base + m.x, (int)m.y, ch,
                                                                          passes);
          }
        }
      }
      events += tick_events;
      if (counts) {
        unsigned long long s = tick_events;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_down_sync(FULL, s, o);
        if (lane == 0 && s) atomicAdd(counts + 2 * (size_t)k + 1, s);
      }
      // 4. Arrive at the grid barrier once the group's list entries and pushes
      //    are issued; thread 0 waits for the other CTAs and announces it.
      group_sync(1, MT);
      if (tid == 0) {
        red_release_add_u32(r.sync, 1u);
        const unsigned target = (unsigned)C * (unsigned)(k + 1) + (unsigned)r.stall_test;
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
        if (ok) {
          cnt_s[k & 3] = (int)__ldcg(r.sync + 1 + m3);
          // Tick t-1's counter has been read by every CTA: clear it for tick t+2.
          if (c == 0) r.sync[1 + (int)((t + 2) % 3)] = 0u;
        } else {
          abort_s = 1;
        }
        mb_arrive(&mb_grid[k & 3]);
      }
      if (warp == 0) __syncwarp(); // warp 0 reconverges after thread 0's wait
    }
  } else {
    // ---------------- delivery group ----------------
    const int dw = warp - MW;
    for (int k = 0; k < ticks; ++k) {
      const long long t = t0 + k;
      const bool bad = !mb_wait(&mb_grid[k & 3], (k >> 2) & 1);
      if (group_any(2, DT, bad || abort_s != 0)) {
        if (tid == MT) {
          if (bad) atomicExch(r.err, 1);
          abort_s = 1;
        }
        break;
      }
      const int S = cnt_s[k & 3], R = (S + 31) >> 5;
      const int *lst = r.lists + (size_t)(t % 3) * d.n_pre;
      const RingAt ra{ring_s, (uint32_t)(2 * P * (int)(t & dr_mask)), (uint32_t)(2 * P * Dr)};
      const LinkQueue links0{link_q, &link_n_s[0], kLinkCap};
      const LinkQueue own_links{warp_q + warp * kWarpLinks, &warp_n_s[warp], kWarpLinks};
      constexpr int D = E::kDepth;
      // This warp's rounds are dw + m*DW, m < M; the blocks of rounds m+1..m+D
      // are in flight while round m is delivered.
      const int M = R > dw ? (R - dw + DW - 1) / DW : 0;
      auto list_at = [&](int m) -> int {
        const int i = (dw + m * DW) * 32 + lane;
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
      // The overflow blocks this warp met, then the group's queue in rounds of 32.
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
      group_sync(2, DT);
      for (int pass = 0; pass < 64; ++pass) {
        const int cur = pass & 1;
        const int n = min(link_n_s[cur], kLinkCap);
        if (n == 0) break;
        const int *q = link_q + cur * kLinkCap;
        const LinkQueue next{link_q + (cur ^ 1) * kLinkCap, &link_n_s[cur ^ 1], kLinkCap};
        for (int rr = dw; rr * 32 < n; rr += DW) {
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
        group_sync(2, DT);
        if (tid == MT) link_n_s[cur] = 0;
        group_sync(2, DT);
      }
      events += tick_events;
      if (counts) {
        unsigned long long s = tick_events;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_down_sync(FULL, s, o);
        if (lane == 0 && s) atomicAdd(counts + 2 * (size_t)k + 1, s);
      }
      __syncwarp();
      if (lane == 0) mb_arrive(&mb_done[k & 3]);
    }
  }

  __syncthreads();
  if (abort_s) return;
  // Write the state back; add the shared ring window [t_end, t_end + Dr) into
  // the global ring (whose slot t_end already holds the last tick's delay-1 pushes).
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
        int2 x = __ldcg(g);
        x.x += q.x;
        x.y += q.y;
        __stcg(g, x);
      }
    }
  }
  const unsigned long long ev = block_sum(events, red_s);
  const unsigned long long sp = block_sum(spikes, red_s);
  if (tid == 0) {
    d.totals[kTotalsStride * (size_t)c] += sp;
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

// Whether entry e of `pre` goes into an owner block: a non-zero weight, and
// (pipelined tick) a delay of at least 2, since delay-1 synapses are pushed by
// the spiking neuron's CTA.
template <bool BSR, bool HALF>
__device__ __forceinline__ bool owner_event(const NetDev &d, const ResidentDev &r, int pre, long long e) {
  if (is_zero<HALF>(edge_weight<BSR, HALF>(d, pre, e))) return false;
  return !r.pipe || (edge_word<BSR>(d, e) >> 28) != 0u;
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
    if (owner_event<BSR, HALF>(d, r, pre, e))
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
// words) and allocates the row's overflow blocks from `cursor` as one run,
// the owner CTAs' chains in CTA order, so that the overflow blocks of a
// spiking row, read by all its owner CTAs in the same tick, lie side by side
// in memory as its primary blocks do.
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
    if (owner_event<BSR, HALF>(d, r, pre, e))
      atomicAdd(&cnt[(int)(edge_word<BSR>(d, e) & kPostMask) / P], 1);
  __syncthreads();
  if (threadIdx.x < 32) {
    // chain[q] = overflow blocks of owners before q (exclusive scan), then one allocation.
    const int lane = threadIdx.x;
    unsigned long long run = 0;
    for (int q0 = 0; q0 < C; q0 += 32) {
      const int q = q0 + lane;
      const int m = q < C ? chain_blocks(cnt[q]) : 0;
      int incl = m;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      if (q < C) chain[q] = (long long)run + (incl - m);
      run += (unsigned long long)__shfl_sync(0xffffffffu, incl, 31);
    }
    unsigned long long b = 0;
    if (lane == 0 && run) b = atomicAdd(cursor, run);
    b = __shfl_sync(0xffffffffu, b, 0);
    const bool fits = b + run <= capacity;
    if (lane == 0 && run && !fits) atomicExch(err, 2);
    for (int q = lane; q < C; q += 32)
      chain[q] = (chain_blocks(cnt[q]) && fits) ? (long long)(primary + b) + chain[q] : -1;
  }
  __syncthreads();
  for (long long e = e0 + threadIdx.x; e < e1; e += BT) {
    if (!owner_event<BSR, HALF>(d, r, pre, e)) continue;
    const uint32_t wb = edge_weight<BSR, HALF>(d, pre, e);
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

// The kernel of this plan: serial or pipelined, 32- or 64-bit events, CSR or
// block storage (pipelined delay-1 push), membrane group of 8 or 16 warps.
void *resident_kernel(const ResidentDev &r, bool bsr) {
  if (!r.pipe)
    return r.ev64 ? reinterpret_cast<void *>(&k_net_resident<Ev64>) : reinterpret_cast<void *>(&k_net_resident<Ev32>);
  const bool wide = r.member_warps == 16;
  if (bsr)
    return wide ? reinterpret_cast<void *>(&k_net_pipe<Ev32, true, 16>) : reinterpret_cast<void *>(&k_net_pipe<Ev32, true, 8>);
  if (r.ev64)
    return wide ? reinterpret_cast<void *>(&k_net_pipe<Ev64, false, 16>) : reinterpret_cast<void *>(&k_net_pipe<Ev64, false, 8>);
  return wide ? reinterpret_cast<void *>(&k_net_pipe<Ev32, false, 16>) : reinterpret_cast<void *>(&k_net_pipe<Ev32, false, 8>);
}

} // namespace

size_t resident_smem_bytes(const ResidentDev &r) {
  const size_t P = size_t(r.per_cta);
  size_t b = size_t(r.ring_depth) * P * 8 + P * 20 + (P / 32) * 4 + 2 * size_t(kLinkCap) * 4 +
             size_t(RW) * kWarpLinks * 4;
  // Pipelined: delay-1 segment of each held neuron (8 bytes, 8-byte aligned).
  if (r.pipe) b = ((b + 7) & ~size_t(7)) + P * 8;
  return b;
}

int resident_max_ctas(const ResidentDev &r, bool bsr, size_t smem) {
  void *fn = resident_kernel(r, bsr);
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
  void *fn = resident_kernel(r, d.bsr != 0);
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
