// Isolated-tick spiking network kernels for sm_100a.
//
// One tick: every neuron reads and clears its delay-ring slot t%16, advances
// its conductance ALIF state (neurogen/biology.py:132-180, frozen synapses),
// and the warp ballots its 32 spike bits into one bitmask word; then the
// outgoing synapses of every spiking neuron are pushed into ring slots
// (t + d) % 16 with integer atomics.  Delays are 1..15, so no push of tick t
// touches slot t%16, and the launch boundary orders tick t's deliveries before
// tick t+1 reads its slot.
//
// Two launch shapes, identical arithmetic:
//   fused  -- one kernel per tick; the warp that owns a spiking neuron pushes
//             its synapses.  Cheapest for small networks (one launch).
//   split  -- k_net_alif updates the neurons and writes the bitmask; then
//             k_net_push CTA b reads the 8 (or 64) bitmask words of its span,
//             lists its spiking neurons (CSR) or non-empty 16-neuron
//             block-columns (block storage) in shared memory, and its 8 warps
//             take the items round-robin, each lane with all of its synapse
//             loads in flight before its deliveries.  For large networks.
// Spike and event counts accumulate into one counter pair per 256-neuron
// group, so the hot path has no same-address atomics.
//
// The neuron arithmetic and its numerics contract are in net_device.cuh.
#include "net_device.cuh"

namespace ngb {
namespace {

constexpr int TB = 256; // threads per block (8 warps)
constexpr int WARPS = TB / 32;

using namespace netdev;

// Membrane update of held neuron i at tick t: reads and clears its ring slot.
__device__ __forceinline__ bool alif_update(const NetDev &d, long long t, int i) {
  const int slot = (int)(t & (kRingSlots - 1));
  int2 *rp = d.ring + (size_t)slot * d.n + i;
  const int2 r = *rp;
  *rp = make_int2(0, 0);
  float v = d.v[i], a = d.a[i], ge = d.ge[i], gi = d.gi[i];
  int ref = d.ref[i];
  const bool s = alif_math(d, t, d.base + i, r, v, a, ge, gi, ref);
  d.v[i] = v;
  d.a[i] = a;
  d.ge[i] = ge;
  d.gi[i] = gi;
  d.ref[i] = ref;
  return s;
}

__device__ __forceinline__ int deliver(const NetDev &d, long long t, uint32_t word, float w) {
  if (w == 0.f) return 0;
  const int post = (int)(word & kPostMask);
  const int dly = (int)(word >> 28) + 1;
  const int slot = (int)((t + dly) & (kRingSlots - 1));
  atomicAdd(reinterpret_cast<int *>(d.ring) + ((size_t)slot * d.n + post) * 2 + (w < 0.f ? 1 : 0), quantum(w));
  return 1;
}

// Push all outgoing CSR synapses of `pre` with the whole warp: each lane takes
// CH (8 or 16) consecutive synapses per pass (16-byte index and weight loads),
// issued together and streamed past the caches (evict-first) before any
// delivery; 8 suits short rows (more lanes busy), 16 long ones (more loads in
// flight a lane).  Rows are padded to multiples of 8 and the arrays carry 16
// spare entries, so the loads stay in bounds; the deliveries are masked to the
// row.  seg selects the whole row (0), its delay-1 segment (1) or the rest (2).
// Returns this lane's delivered (non-zero) synapse count.
template <int CH>
__device__ __forceinline__ int push_row(const NetDev &d, long long t, int pre, int lane, int seg) {
  long long e0 = d.row[pre], e1 = d.row[pre + 1];
  if (seg == 1) e1 = e0 + d.mid[pre];
  else if (seg == 2) e0 += d.mid[pre];
  int delivered = 0;
  for (long long e = e0 + lane * CH; e < e1; e += 32 * CH) {
    const uint4 *ps = reinterpret_cast<const uint4 *>(d.syn + e);
    uint4 p[CH / 4];
#pragma unroll
    for (int q = 0; q < CH / 4; ++q) p[q] = __ldcs(ps + q);
    float w[CH];
    if (d.w_half) {
      const uint4 *pw = reinterpret_cast<const uint4 *>(static_cast<const __half *>(d.w) + e);
#pragma unroll
      for (int q = 0; q < CH / 8; ++q) {
        const uint4 wv = __ldcs(pw + q);
        const uint32_t h[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          w[8 * q + 2 * j] = half_bits(h[j] & 0xFFFFu);
          w[8 * q + 2 * j + 1] = half_bits(h[j] >> 16);
        }
      }
    } else {
      const float4 *pw = reinterpret_cast<const float4 *>(static_cast<const float *>(d.w) + e);
#pragma unroll
      for (int q = 0; q < CH / 4; ++q) {
        const float4 f = __ldcs(pw + q);
        w[4 * q] = f.x; w[4 * q + 1] = f.y; w[4 * q + 2] = f.z; w[4 * q + 3] = f.w;
      }
    }
#pragma unroll
    for (int q = 0; q < CH / 4; ++q) {
      const uint32_t word[4] = {p[q].x, p[q].y, p[q].z, p[q].w};
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (e + 4 * q + j < e1) delivered += deliver(d, t, word[j], w[4 * q + j]);
    }
  }
  return delivered;
}

// Push the spiking columns `sub` (16-bit mask) of block-column bc: each lane
// takes one block at a time, sums the selected tile columns per post row in
// fixed point (E and I apart), and issues one atomic per non-zero row sum.
__device__ __forceinline__ int push_block_column(const NetDev &d, long long t, int bc, unsigned sub, int lane,
                                                 int seg) {
  long long b0 = d.bcol[bc], b1 = d.bcol[bc + 1];
  if (seg == 1) b1 = b0 + d.bmid[bc];
  else if (seg == 2) b0 += d.bmid[bc];
  int delivered = 0;
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
          delivered += w != 0.f;
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
  return delivered;
}

// CTA-wide sum of one value per warp (lane 0 contributes), added to this
// group's running counter (single writer) and, when given, to this tick's
// counter (recording runs only).
__device__ __forceinline__ void add_block_count(unsigned long long v, unsigned long long *group_total,
                                                unsigned long long *tick_count) {
  __shared__ unsigned long long part[WARPS];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
  if (lane == 0) part[warp] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long s = 0;
    for (int k = 0; k < WARPS; ++k) s += part[k];
    *group_total += s;
    if (tick_count && s) atomicAdd(tick_count, s);
  }
  __syncthreads();
}

template <bool BSR>
__global__ void __launch_bounds__(TB) k_net_fused(NetDev d, TickRef tr, uint32_t *spikes_out,
                                                  unsigned long long *counts) {
  const long long t = tick_of(tr);
  const int i = blockIdx.x * TB + threadIdx.x;
  const int lane = threadIdx.x & 31;
  const bool s = i < d.n ? alif_update(d, t, i) : false;
  const unsigned fired = __ballot_sync(0xffffffffu, s);
  const int base = i - lane; // fused launches are unpartitioned: base 0
  if (lane == 0 && base < d.n) {
    d.bitmask[(t % d.bm_bufs) * d.bm_stride + (base >> 5)] = fired;
    if (spikes_out) spikes_out[base >> 5] = fired;
  }
  unsigned long long events = 0;
  if (BSR) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const unsigned sub = (fired >> (16 * half)) & 0xFFFFu;
      if (sub) events += push_block_column(d, t, (base >> 4) + half, sub, lane, 0);
    }
  } else {
    unsigned m = fired;
    while (m) {
      const int src = __ffs(m) - 1;
      m &= m - 1;
      events += push_row<16>(d, t, base + src, lane, 0);
    }
  }
  unsigned long long *group = d.totals + kTotalsStride * (size_t)blockIdx.x;
  add_block_count(lane == 0 ? __popc(fired) : 0, group, counts);
  add_block_count(events, group + 1, counts ? counts + 1 : nullptr);
}

template <bool BSR>
__global__ void __launch_bounds__(TB) k_net_alif(NetDev d, TickRef tr, uint32_t *spikes_out,
                                                 unsigned long long *counts) {
  const long long t = tick_of(tr);
  const int i = blockIdx.x * TB + threadIdx.x;
  const int lane = threadIdx.x & 31;
  const bool s = i < d.n ? alif_update(d, t, i) : false;
  if (d.rate && i < d.n) {
    // Learning networks: the rate trace (biology.py:167-168), and from it this
    // tick's synaptic-scaling factor of the neuron's E contacts (:207-208),
    // exp(clip((target - rate) / target * dt / tau, -.001, .001)).
    float r = __fmul_rn(d.rate[i], d.l_slow);
    if (s) r = __fadd_rn(r, d.l_rate_inc);
    d.rate[i] = r;
    float x = __fdiv_rn(__fmul_rn(__fdiv_rn(__fsub_rn(d.l_target, r), d.l_target), d.l_dt), d.l_tau_s);
    x = x < -.001f ? -.001f : (x > .001f ? .001f : x);
    d.scale[i] = ng_expf(x);
  }
  const unsigned fired = __ballot_sync(0xffffffffu, s);
  const int base = i - lane;
  __shared__ uint32_t words_s[WARPS];
  if (lane == 0 && base < d.n) {
    if (d.peer_bm) words_s[threadIdx.x >> 5] = fired;
    else d.bitmask[(size_t)(t % d.bm_bufs) * d.bm_stride + ((d.base + base) >> 5)] = fired;
    if (d.hist) d.hist[(t & (kRingSlots - 1)) * d.bm_stride + (base >> 5)] = fired;
    if (spikes_out) spikes_out[base >> 5] = fired;
  }
  add_block_count(lane == 0 ? __popc(fired) : 0, d.totals + kTotalsStride * (size_t)blockIdx.x, counts);
  if (d.peer_bm) {
    // The CTA's words (after the barrier in add_block_count) into every
    // rank's buffer: thread j stores word j % WARPS to rank j / WARPS, so each
    // rank gets one contiguous 32-byte piece; each storing thread fences its
    // store system-wide before the CTA ends (k_net_xwait raises the flags
    // once the whole kernel has ended).
    const int j = threadIdx.x, w = j % WARPS, r = j / WARPS;
    const int first = blockIdx.x * TB + w * 32;
    if (r < d.world && first < d.n) {
      d.peer_bm[r][(size_t)(t % d.bm_bufs) * d.bm_stride + ((d.base + first) >> 5)] = words_s[w];
      __threadfence_system();
    }
  }
}

// Runs after this rank's k_net_alif of tick t has ended (stream order), whose
// threads fenced their stores system-wide: lane r raises this rank's flag in
// rank r, then waits for rank r's flag here.
__global__ void k_net_xwait(NetDev d, TickRef tr) {
  const long long t = tick_of(tr);
  const int r = threadIdx.x;
  if (r >= d.world || *(volatile int *)d.xerr) return;
  const unsigned long long target = (*d.xepoch << 40) | ((unsigned long long)t + 1ull);
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(d.peer_flag[r] + d.rank), "l"(target) : "memory");
  unsigned long long start;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(start));
  for (unsigned spin = 0; spin < (1u << 30); ++spin) {
    unsigned long long f;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(f) : "l"(d.xflag + r) : "memory");
    if (f >= target) return;
    if ((spin & 63u) == 63u) {
      unsigned long long now;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
      if (now - start > 2000000000ull || *(volatile int *)d.xerr) break;
    }
  }
  atomicExch(d.xerr, 1);
}


// ---------------------------------------------------------------------------
// Learning (plasticity networks): biology.py:182-218 in the fp32 contract of
// oracle/net_oracle.c (learn32): every operation rounded as written, the
// constants the reference's expressions in double rounded once.  One warp per
// presynaptic row: lanes 0..15 read the row's spike bit of the last 16 ticks
// from the history (bit j: tick t - j), so a contact of delay d sees its
// arrival as bit d; the lanes then take the row's contacts 32 at a time.
// Zero-weight entries (row padding) are not contacts.  The post trace of every
// neuron is decayed and advanced after all contacts have read it, by the
// tick's push (k_net_push, whole rows).
// ---------------------------------------------------------------------------
// One contact's learning step (the fp32 contract); a = arrival, post = postsynaptic spike.
// A stored contact's potential arrival is its arrival (biology.py:141-146 for
// an active contact), so its potential trace equals its pre trace at every
// tick: one array holds both.
__device__ __forceinline__ void learn_contact(const NetDev &d, bool exc, int q, float a, float post, float &w_io,
                                              float &pre_tr, float &coact, float &usage) {
  const float pt = __fmul_rn(pre_tr, d.l_decay);
  const float pot = pt;
  const float pq = __fmul_rn(d.post_tr[q], d.l_decay);
  float w = fabsf(w_io);
  if (d.learn_weights) {
    float delta;
    if (exc) {
      delta = __fmul_rn(d.l_stdp, __fsub_rn(__fmul_rn(__fmul_rn(pt, post), __fsub_rn(4.f, w)),
                                            __fmul_rn(__fmul_rn(__fmul_rn(1.05f, pq), a), w)));
    } else {
      delta = __fmul_rn(d.l_inh, __fadd_rn(__fmul_rn(a, __fsub_rn(pq, d.l_alpha)), __fmul_rn(pt, post)));
      delta = __fmul_rn(delta, q < d.n_exc ? 1.f : 0.f);
    }
    w = __fadd_rn(w, delta);
    if (exc) w = __fmul_rn(w, d.scale[q]); // the postsynaptic neuron's factor (k_net_alif)
    const float hi = exc ? 4.f : 12.f;
    w = w < .01f ? .01f : w;
    w = w > hi ? hi : w;
  }
  coact = __fadd_rn(__fmul_rn(coact, d.l_slow), __fmul_rn(__fmul_rn(d.l_oms, pot), post));
  usage = __fadd_rn(__fmul_rn(usage, d.l_slow), __fmul_rn(__fmul_rn(d.l_oms, a), d.l_per_ms));
  pre_tr = __fadd_rn(pt, a);
  w_io = w_io < 0.f ? -w : w;
}

__global__ void __launch_bounds__(TB) k_net_learn(NetDev d, TickRef tr) {
  const long long t = tick_of(tr);
  const int lane = threadIdx.x & 31, hl = lane & 15;
  // Two presynaptic rows a warp, one a half-warp.
  const int p = (blockIdx.x * WARPS + (threadIdx.x >> 5)) * 2 + (lane >> 4);
  const bool valid = p < d.n_pre;
  uint32_t bit = 0;
  if (valid) bit = (d.hist[((t - hl) & (kRingSlots - 1)) * d.bm_stride + (p >> 5)] >> (p & 31)) & 1u;
  // bit j of `past`: the row's spike at tick t - j (j < 16).
  const unsigned past = (__ballot_sync(0xffffffffu, bit != 0) >> (lane & 16)) & 0xFFFFu;
  if (!valid) return;
  const uint32_t *now = d.hist + (t & (kRingSlots - 1)) * d.bm_stride;
  const bool exc = p < d.n_exc;
  float *w32 = static_cast<float *>(const_cast<void *>(d.w));
  // Rows start and end on multiples of 8 entries: four contacts a lane, 16-byte accesses.
  const long long e1 = d.row[p + 1];
  for (long long e = d.row[p] + 4 * hl; e < e1; e += 64) {
    float4 w4 = *reinterpret_cast<const float4 *>(w32 + e);
    if (w4.x == 0.f && w4.y == 0.f && w4.z == 0.f && w4.w == 0.f) continue; // row padding
    const uint4 s4 = *reinterpret_cast<const uint4 *>(d.syn + e);
    float4 pr = *reinterpret_cast<const float4 *>(d.pre_tr + e);
    float4 co = *reinterpret_cast<const float4 *>(d.coact + e);
    float4 us = *reinterpret_cast<const float4 *>(d.usage + e);
    float *wv = &w4.x, *prv = &pr.x, *cov = &co.x, *usv = &us.x;
    const uint32_t words[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (wv[j] == 0.f) continue; // not a contact
      const int q = (int)(words[j] & kPostMask);
      const int dly = (int)(words[j] >> 28) + 1;
      const float a = ((past >> dly) & 1u) ? 1.f : 0.f;
      const float post = ((now[q >> 5] >> (q & 31)) & 1u) ? 1.f : 0.f;
      learn_contact(d, exc, q, a, post, wv[j], prv[j], cov[j], usv[j]);
    }
    *reinterpret_cast<float4 *>(w32 + e) = w4;
    *reinterpret_cast<float4 *>(d.pre_tr + e) = pr;
    *reinterpret_cast<float4 *>(d.coact + e) = co;
    *reinterpret_cast<float4 *>(d.usage + e) = us;
  }
}


// CTA b pushes the spikes of presynaptic neurons [32*SPANW*b, 32*SPANW*(b+1)):
// warp 0 lists them from the span's SPANW bitmask words (block storage: 8
// words, listed by 16-neuron block-column) and the warps take them round-
// robin.  Wide spans (64 words) keep the grid proportional to the work when
// the presynaptic population is large and each rank's share of a row short.
// SEG selects whole rows (0), delay-1 segments (1) or delay>=2 segments (2).
template <bool BSR, int SEG, int SPANW, int CH>
__global__ void __launch_bounds__(TB) k_net_push(NetDev d, TickRef tr, unsigned long long *counts) {
  static_assert(!BSR || SPANW == 8, "block storage scans 8 words a CTA");
  constexpr int SPAN = 32 * SPANW;
  __shared__ int items[SPAN];
  __shared__ unsigned item_mask[BSR ? SPAN / 16 : 1];
  __shared__ int n_items;
  const long long t = tick_of(tr);
  const uint32_t *bitmask = d.bitmask + (t % d.bm_bufs) * d.bm_stride;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int base = blockIdx.x * SPAN;
  if (SEG == 0 && d.post_tr) {
    // Learning networks: the post traces of this span's neurons, decayed and
    // advanced by this tick's spikes once every contact has read them
    // (k_net_learn, the previous launch).
    for (int i = base + threadIdx.x; i < min(base + SPAN, d.n); i += TB) {
      const float sp = ((bitmask[i >> 5] >> (i & 31)) & 1u) ? 1.f : 0.f;
      d.post_tr[i] = __fadd_rn(__fmul_rn(d.post_tr[i], d.l_decay), sp);
    }
  }
  if (warp == 0) {
    if (BSR) {
      const int w = base / 32 + (lane & 7);
      const unsigned word = (lane < 8 && base + (lane & 7) * 32 < d.n_pre) ? bitmask[w] : 0u;
      // 16 block-columns per group; lane k < 16 owns half (k & 1) of word k / 2.
      const unsigned wk = __shfl_sync(0xffffffffu, word, (lane >> 1) & 7);
      const unsigned sub = lane < 16 ? ((wk >> (16 * (lane & 1))) & 0xFFFFu) : 0u;
      const unsigned has = __ballot_sync(0xffffffffu, sub != 0);
      if (sub) {
        const int at = __popc(has & ((1u << lane) - 1u));
        items[at] = (base >> 4) + lane;
        item_mask[at] = sub;
      }
      if (lane == 0) n_items = __popc(has);
    } else {
      // Lane l reads words l and l + 32 of the span (those that exist).
      const unsigned w0 = (lane < SPANW && base + lane * 32 < d.n_pre) ? bitmask[base / 32 + lane] : 0u;
      const unsigned w1 = (lane + 32 < SPANW && base + (lane + 32) * 32 < d.n_pre) ? bitmask[base / 32 + lane + 32] : 0u;
      const unsigned cnt = __popc(w0) + __popc(w1);
      unsigned pre = cnt; // inclusive scan over the lanes
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned v = __shfl_up_sync(0xffffffffu, pre, o);
        if (lane >= o) pre += v;
      }
      unsigned at = pre - cnt;
      for (unsigned m = w0; m; m &= m - 1) items[at++] = base + lane * 32 + (__ffs(m) - 1);
      for (unsigned m = w1; m; m &= m - 1) items[at++] = base + (lane + 32) * 32 + (__ffs(m) - 1);
      if (lane == 31) n_items = (int)pre;
    }
  }
  __syncthreads();
  const int count = n_items;
  unsigned long long events = 0;
  for (int k = warp; k < count; k += WARPS) {
    if (BSR) events += push_block_column(d, t, items[k], item_mask[k], lane, SEG);
    else events += push_row<CH>(d, t, items[k], lane, SEG);
  }
  add_block_count(events, d.totals + kTotalsStride * (size_t)blockIdx.x + (SEG == 2 ? 2 : 1),
                  counts ? counts + 1 : nullptr);
}

__global__ void k_set_tick(long long *t, long long v) { *t = v; }
__global__ void k_add_tick(long long *t, long long dv) { *t += dv; }

} // namespace

void launch_net_fused(const NetDev &d, TickRef t, uint32_t *spikes_out, unsigned long long *counts,
                      cudaStream_t s) {
  const int blocks = (d.n + TB - 1) / TB;
  if (d.bsr) k_net_fused<true><<<blocks, TB, 0, s>>>(d, t, spikes_out, counts);
  else k_net_fused<false><<<blocks, TB, 0, s>>>(d, t, spikes_out, counts);
}

void launch_net_alif(const NetDev &d, TickRef t, uint32_t *spikes_out, unsigned long long *counts,
                     cudaStream_t s) {
  const int blocks = (d.n + TB - 1) / TB;
  if (d.bsr) k_net_alif<true><<<blocks, TB, 0, s>>>(d, t, spikes_out, counts);
  else k_net_alif<false><<<blocks, TB, 0, s>>>(d, t, spikes_out, counts);
}

void launch_net_xwait(const NetDev &d, TickRef t, cudaStream_t s) { k_net_xwait<<<1, 32, 0, s>>>(d, t); }

void launch_net_learn(const NetDev &d, TickRef t, cudaStream_t s) {
  if (d.n_pre > 0) k_net_learn<<<(d.n_pre + 2 * WARPS - 1) / (2 * WARPS), TB, 0, s>>>(d, t);
}

template <bool BSR, int SPANW, int CH>
void push_seg(const NetDev &d, TickRef t, unsigned long long *counts, int seg, cudaStream_t s) {
  const int span = 32 * SPANW, blocks = (d.n_pre + span - 1) / span;
  if (seg == 1) k_net_push<BSR, 1, SPANW, CH><<<blocks, TB, 0, s>>>(d, t, counts);
  else if (seg == 2) k_net_push<BSR, 2, SPANW, CH><<<blocks, TB, 0, s>>>(d, t, counts);
  else k_net_push<BSR, 0, SPANW, CH><<<blocks, TB, 0, s>>>(d, t, counts);
}

void launch_net_push(const NetDev &d, TickRef t, unsigned long long *counts, int seg, cudaStream_t s) {
  if (d.bsr) return push_seg<true, 8, 16>(d, t, counts, seg, s);
  if (d.push_span_words == 64) {
    if (d.push_chunk == 8) return push_seg<false, 64, 8>(d, t, counts, seg, s);
    return push_seg<false, 64, 16>(d, t, counts, seg, s);
  }
  if (d.push_chunk == 8) return push_seg<false, 8, 8>(d, t, counts, seg, s);
  return push_seg<false, 8, 16>(d, t, counts, seg, s);
}

void launch_set_tick(long long *t_dev, long long value, cudaStream_t s) { k_set_tick<<<1, 1, 0, s>>>(t_dev, value); }
void launch_add_tick(long long *t_dev, long long delta, cudaStream_t s) { k_add_tick<<<1, 1, 0, s>>>(t_dev, delta); }

} // namespace ngb
