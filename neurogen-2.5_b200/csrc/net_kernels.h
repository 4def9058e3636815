// Launch interface of the isolated-tick network kernels (net_kernels.cu).
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace ngb {

constexpr int kRingSlots = 16; // delay ring depth; delays 1..15 ticks
constexpr float kRingQuantum = 5.9604644775390625e-08f; // 2^-24 nS per ring unit
constexpr int kRowPad = 8;     // CSR rows padded to multiples of 8 synapses
constexpr int kTailPad = 16;   // extra zero synapses after the last row

// Synapse word: postsynaptic index in bits 0-27, (delay - 1) in bits 28-31.
constexpr uint32_t kPostMask = 0x0FFFFFFFu;

struct NetDev {
  int n, n_exc;  // n: neurons held here (state, ring); n_exc: global E/I split
  int n_pre;     // presynaptic rows = neurons of the whole network
  int base;      // global index of the first neuron held here (multiple of 32)
  // CSR by presynaptic neuron, rows padded to multiples of 8 with zero weights.
  const long long *row; // [n+1]
  const uint32_t *syn;  // packed post/delay
  const void *w;        // fp16 or fp32 signed weights (nS; negative = inhibitory)
  int w_half;
  const int *outdeg; // non-zero synapses per presynaptic neuron
  const int *mid;    // per row: offset of its delay>=2 segment (delay-1 synapses first)
  // 16x16 block storage by block-column (pre block), blocks sorted by block-row.
  int bsr;
  const long long *bcol; // [n/16+1]
  const uint32_t *blk;   // block-row | (delay-1) << 28
  const uint16_t *tiles; // fp16 [block][16 pre columns][16 post rows]
  const int *bmid;       // per block-column: number of its delay-1 blocks (first)
  // State (fp32 SoA) and the E/I delay ring [16][n] of int2 (E, I) in 2^-24 nS.
  float *v, *a, *ge, *gi;
  int *ref;
  int2 *ring;
  uint32_t *bitmask;            // spike words of the whole network, bm_bufs buffers (by t % bm_bufs)
  int bm_stride;                // words per buffer
  int bm_bufs;                  // 2; 3 with the peer exchange
  // Peer exchange of a partitioned network (one-sided, over NVLink; null:
  // NCCL all-gather): every rank's bitmask buffers and flag array mapped here
  // ([world], this rank's own at [rank]); flag[r] = 1 + the last tick whose
  // whole slice rank r has stored into this rank's buffers, in the low 40 bits;
  // the exchange epoch (advanced by every collective ng_net_set_state) above.
  uint32_t *const *peer_bm;
  unsigned long long *const *peer_flag;
  unsigned long long *xflag;    // this rank's flag array [world]
  int *xerr;                    // 1: a wait for a peer's flag ran out
  const unsigned long long *xepoch; // the exchange epoch (device memory, read by the kernels)
  int world, rank;
  int push_span_words;          // split push: bitmask words a CTA scans (8 or 64)
  int push_chunk;               // split push: synapses a lane takes a pass (8 or 16)
  // Running counters since creation, three per 256-neuron group: [g][0]
  // spikes of held group g (membrane kernel), [g][1] events pushed from
  // presynaptic group g by the delay-1 (or whole-row) push, [g][2] by the
  // delay>=2 push.  One writer per entry, no atomics.
  unsigned long long *totals;
  // Constants (see net_kernels.cu for the exact operation order).
  float dE, dI, dA, g_leak, gLEL, e_inh, v_th, v_reset, cap_e, cap_i, neg_dt, adapt_inc, bias,
      drive_ns;
  int drive_kind; // 0 conductance events, 1 imposed spikes
  uint32_t drive_thr;
  unsigned long long drive_key;
  int ref_ticks;
  // Learning (plasticity networks; null pointers otherwise): per CSR entry the
  // pre trace (equal to the potential trace for a stored contact), coactivity
  // and usage; per neuron the post trace and the rate; the spike bitmask of the
  // last kRingSlots ticks [16][bm_stride].
  float *pre_tr, *coact, *usage, *post_tr, *rate;
  float *scale;   // per neuron, this tick: the synaptic-scaling factor of its E contacts
  uint32_t *hist;
  int learn_weights; // 1: weights learn (0: traces only)
  // Constants of the fp32 contract (the reference's expressions in double, rounded once).
  float l_decay, l_slow, l_oms, l_rate_inc, l_per_ms, l_alpha, l_stdp, l_inh, l_target, l_tau_s, l_dt;
};

// Which tick a launch computes: *t_dev + k when t_dev is set (graph replay
// with a device-resident tick counter), else k.
struct TickRef {
  const long long *t_dev;
  long long k;
};

// Fused single launch per tick (small networks): ALIF, ballot, push.
void launch_net_fused(const NetDev &d, TickRef t, uint32_t *spikes_out, unsigned long long *counts,
                      cudaStream_t s);
// Split path (large networks): ALIF + bitmask, then the push of the spikes of
// each 256-neuron group by one CTA.
void launch_net_alif(const NetDev &d, TickRef t, uint32_t *spikes_out, unsigned long long *counts,
                     cudaStream_t s);
// Peer exchange: wait (bounded, 2 s) until every rank's slice of tick t has
// arrived; on a timeout *xerr = 1 and later waits return at once.
void launch_net_xwait(const NetDev &d, TickRef t, cudaStream_t s);
// seg: 0 whole rows, 1 delay-1 segments only, 2 delay>=2 segments only.
void launch_net_push(const NetDev &d, TickRef t, unsigned long long *counts, int seg, cudaStream_t s);
// Learning of tick t (plasticity networks), after k_net_alif and before the
// push: every contact's weight and traces (biology.py:182-218).  The push of
// the tick (whole rows) then advances every neuron's post trace.
void launch_net_learn(const NetDev &d, TickRef t, cudaStream_t s);
constexpr int kTotalsStride = 3;
constexpr int kNetBlock = 256; // neurons per membrane CTA
void launch_set_tick(long long *t_dev, long long value, cudaStream_t s);
void launch_add_tick(long long *t_dev, long long delta, cudaStream_t s);

// Resident launch shape (net_resident.cu): a persistent cooperative launch
// runs many ticks with CTA c owning neurons [c*per_cta, (c+1)*per_cta), their
// state and a ring of ring_depth slots in shared memory.
constexpr int kResidentThreads = 1024;
constexpr int kOwnerBlockSlots = 8; // event words per owner block
constexpr int kResidentPipeDefault = 0; // resident tick by default: 0 serial, 1 pipelined
struct ResidentDev {
  int ctas;           // C (all co-resident)
  int per_cta;        // P, a multiple of 32, at most 2048
  int ring_depth;     // Dr: power of two >= the largest delay; 2*(Dr+1)*P < 2^16
  int ev64;           // 1: 64-bit events (fp32 weights), 0: 32-bit (fp16)
  int stall_test;     // failure-path tests only: 1 makes the first barrier wait run out
  // 0: serial tick (membrane, list, barrier, delivery of every synapse in turn);
  // 1: pipelined tick (delay-1 synapses pushed into the global ring by the
  //    spiking neuron's CTA; owner blocks hold delay>=2 synapses only and are
  //    delivered by a warp group while the membrane warps run the next tick).
  int pipe;
  int member_warps;   // pipelined: warps of the membrane group (8 or 16)
  const void *blocks; // [n_pre][C] owner blocks of 8 events, then overflow blocks
  int *lists;         // [3][n_pre] spike ids of the tick (serial: by parity; pipelined: by t%3)
  unsigned *sync;     // [0] grid barrier counter, [1 + t%3] list length of tick t;
                      // zeroed before each launch
  int *err;           // set to 1 by a barrier timeout
};
size_t resident_smem_bytes(const ResidentDev &r);
// Co-resident CTAs of the plan's kernel at this shared-memory size (0: none).
int resident_max_ctas(const ResidentDev &r, bool bsr, size_t smem);
// ticks ticks from tick t0; spikes_out [ticks][words] and counts [ticks][2] optional.
cudaError_t launch_net_resident(const NetDev &d, const ResidentDev &r, long long t0, int ticks, uint32_t *spikes_out,
                                unsigned long long *counts, int words, cudaStream_t s);
// Owner-block construction from the device CSR: overflow blocks needed
// (added to *need), then the blocks themselves (array pre-filled with all-ones
// words; overflow blocks taken from *cursor; *err = 2 past `capacity`).
void launch_owner_count(const NetDev &d, const ResidentDev &r, unsigned long long *need, cudaStream_t s);
void launch_owner_fill(const NetDev &d, const ResidentDev &r, void *blocks, unsigned long long *cursor,
                       unsigned long long capacity, int *err, cudaStream_t s);

// Fixed fan-in synapses drawn on the device for held posts [lo, lo + np) of an
// n-neuron network (net_generate.cu), fp16 weights.  Keys are the host
// generator's stream keys.
struct FaninGen {
  int n, n_exc, lo, np, fanin, delay_min, delay_span;
  float sigma;
  unsigned long long key_pre, key_delay, key_w1, key_w2;
};
// c1/c2[pre] += delay-1 / delay>=2 synapses of row pre.
void launch_fanin_count(const FaninGen &g, int *c1, int *c2, cudaStream_t s);
// Writes syn/w16 at row[pre] (+ mid[pre] for delay>=2) through the cursors;
// *bad_post = lowest held post whose input can overflow the ring (else unchanged).
void launch_fanin_fill(const FaninGen &g, const long long *row, const int *mid, int *cur1, int *cur2, uint32_t *syn,
                       uint16_t *w16, int *bad_post, cudaStream_t s);

} // namespace ngb
