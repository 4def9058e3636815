// Host side of the isolated-tick spiking network: topology generation, device
// layout (CSR or 16x16 blocks by presynaptic neuron), state and tick loop.
#pragma once
#include "common.h"
#include "net_kernels.h"
#include "nccl_dl.h"
#include "neurogen_b200.h"

#include <cstdint>
#include <mutex>
#include <vector>

namespace ngb {

// Synapses by presynaptic neuron, host form.
struct HostCSR {
  int n = 0;                     // presynaptic rows (all neurons of the network)
  int post_base = 0, n_post = 0; // postsynaptic neurons held: [post_base, post_base + n_post)
  std::vector<long long> row;    // [n+1], rows padded to multiples of 8
  std::vector<uint32_t> syn;     // (post - post_base) | (delay-1) << 28
  std::vector<float> w32;        // signed weights (fp32 storage), or
  std::vector<uint16_t> w16;     // fp16 bits (fp16 storage)
  std::vector<int> outdeg;       // non-zero synapses per row
  // Offset (from the row start, a multiple of 8) of the row's second segment:
  // rows hold their delay-1 synapses first, then the rest, each segment padded.
  std::vector<int> mid;
};

// 16x16 blocks by block-column, host form.
struct HostBSR {
  int nb = 0;                    // block-columns (= block-rows)
  std::vector<long long> bcol;   // [nb+1]
  std::vector<uint32_t> blk;     // block-row | (delay-1) << 28
  std::vector<uint16_t> tiles;   // fp16 [block][16 columns][16 rows]
  std::vector<int> outdeg;       // non-zero synapses per presynaptic neuron
  std::vector<int> mid;          // per block-column: number of its delay-1 blocks (listed first)
};

// Reorders each CSR row (block-column) so that its delay-1 synapses (blocks)
// come first, in their own padded segment; fills `mid`.
void split_by_delay(HostCSR &h);
void split_by_delay(HostBSR &b);

// A generated or caller-given synapse set on the host (no device needed).
struct Topology {
  ng_net_config cfg;
  bool blocks = false; // true: `bsr` holds the synapses, else `csr`
  HostCSR csr;
  HostBSR bsr;
  int64_t synapses() const;
  // Synapse list, presynaptic-major (arrays of synapses() entries; any may be null).
  void export_edges(int32_t *pre, int32_t *post, int32_t *delay, float *weight) const;
};
Topology *make_topology(const ng_net_config &cfg);
Topology *make_topology_edges(const ng_net_config &cfg, int64_t nnz, const int32_t *pre, const int32_t *post,
                              const int32_t *delay, const float *w);

// Deterministic generators (same seed -> same network on any machine).
void generate_csr(const ng_net_config &c, HostCSR &out);
void generate_bsr(const ng_net_config &c, HostBSR &out);
void csr_from_edges(const ng_net_config &c, int64_t nnz, const int32_t *pre, const int32_t *post,
                    const int32_t *delay, const float *w, HostCSR &out);
void validate_config(const ng_net_config &c);

struct DeviceFanin {}; // tag: draw a fixed fan-in network's synapses on the device

class Network {
public:
  // nccl_id: 128-byte NCCL unique id, required when cfg.part_world > 1
  // (collective: every rank constructs its partition at the same time).
  explicit Network(const Topology &topo, const void *nccl_id = nullptr);
  Network(const ng_net_config &cfg, const void *nccl_id, DeviceFanin);
  ~Network();
  Network(const Network &) = delete;
  Network &operator=(const Network &) = delete;

  int64_t synapses() const { return nnz_; }
  void export_edges(int32_t *pre, int32_t *post, int32_t *delay, float *weight);
  void set_state(const float *v, const float *a, const float *ge, const float *gi, const int32_t *ref,
                 const int32_t *ring, int64_t tick);
  void get_state(float *v, float *a, float *ge, float *gi, int32_t *ref, int32_t *ring, int64_t *tick);
  // Enqueue `ticks` ticks on `st`; d_spikes [ticks][words] and d_counts
  // [ticks][2] (u64) are optional device outputs.
  void enqueue(int ticks, uint32_t *d_spikes, unsigned long long *d_counts, cudaStream_t st);
  void run_host(int ticks, uint32_t *spikes, int64_t *counts);
  void stats(int64_t *totals);
  // Learning networks: per-contact traces in export order, per-neuron post trace and rate.
  void plasticity_state(float *pre_tr, float *pot_tr, float *coact, float *usage, float *post_tr, float *rate);
  bool split() const { return split_; }
  int exchange_kind() const { return world_ > 1 ? (dev_.peer_bm ? 2 : 1) : 0; }
  bool resident() const { return resident_; }
  const ResidentDev &resident_plan() const { return res_; }

  ng_net_config cfg;
  int device = 0;
  cudaStream_t stream = nullptr;
  std::mutex mutex;

private:
  int n_ = 0, n_pre_ = 0, base_ = 0, world_ = 1, rank_ = 0;
  size_t totals_pairs_ = 0;
  ncclComm_t comm_ = nullptr;
  int64_t nnz_ = 0;
  long long tick_ = 0;
  NetDev dev_{};
  DeviceBuffer row_, syn_, w_, outdeg_, mid_, bcol_, blk_, tiles_;
  DeviceBuffer v_, a_, ge_, gi_, ref_, ring_;
  DeviceBuffer rec_spikes_, rec_counts_;
  DeviceBuffer bitmask_, totals_, tick_dev_;
  DeviceBuffer pre_tr_, coact_, usage_, post_tr_, rate_, scale_, hist_; // learning
  void init_learning(size_t bm_words);
  // One-sided spike exchange (partitioned networks).
  DeviceBuffer xbuf_, peer_bm_, peer_flag_, xctl_;
  std::vector<void *> peer_bases_;
  void setup_peer_exchange(size_t bm_words);
  void check_exchange();
  void exchange_epoch();
  unsigned long long epoch_ = 0;
  bool split_ = false;
  cudaGraphExec_t graph_ = nullptr;
  static constexpr int kGraphTicks = 64;
  cudaStream_t stream_rest_ = nullptr; // graph replays: delay>=2 pushes beside the next tick
  cudaEvent_t ev_fork_ = nullptr, ev_alif_ = nullptr, ev_rest_[2] = {nullptr, nullptr}, ev_join_ = nullptr;
  void launch_membrane(TickRef t, int parity, uint32_t *spikes_row, unsigned long long *counts_row,
                       cudaStream_t st);
  void launch_tick(TickRef t, int parity, uint32_t *spikes_row, unsigned long long *counts_row, cudaStream_t st);
  void capture_graph();
  // Resident launch: plan, owner blocks, buffers.
  bool resident_ = false;
  ResidentDev res_{};
  DeviceBuffer res_blocks_, res_lists_, res_sync_, res_err_;
  static constexpr int kResidentChunk = 2048; // ticks per persistent launch
  bool plan_resident(int max_delay, bool required);
  void generate_fanin_device(int lo, int hi);
  void init_state(const void *nccl_id, int max_delay);
  void build_owner_blocks();
  void check_resident();
};

} // namespace ngb
