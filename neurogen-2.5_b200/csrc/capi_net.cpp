// C ABI of the isolated-tick spiking network (include/neurogen_b200.h part 4).
#include "capi_common.h"
#include "net_engine.h"
#include "nccl_dl.h"
#include "neurogen_b200.h"

#include <cstring>
#include <memory>
#include <mutex>

using namespace ngb;

extern "C" {

void ng_net_default_config(ng_net_config *c) {
  if (!c) return;
  std::memset(c, 0, sizeof *c);
  c->n = 1024;
  c->n_exc = 819; // first 80% excitatory
  c->topology = NG_TOPO_ERDOS_RENYI;
  c->p_connect = 0.02f;
  c->fanin = 512;
  c->bsr_blocks = 128;
  c->bsr_fill = 64;
  c->weight_kind = NG_W_LOGNORMAL_F32;
  c->w_mu = -2.f;
  c->w_sigma = 0.5f;
  c->delay_min = 1;
  c->delay_max = 8;
  c->seed = 0;
  // BiologyConfig defaults and the membrane constants of biology.py:153-170.
  c->dt_ms = 1.f;
  c->cap_exc_pf = 200.f;
  c->cap_inh_pf = 100.f;
  c->g_leak_ns = 10.f;
  c->e_leak_mv = -65.f;
  c->e_inh_mv = -80.f;
  c->v_thresh_mv = -50.f;
  c->v_reset_mv = -65.f;
  c->t_ref_ms = 2.f;
  c->tau_exc_ms = 5.f;
  c->tau_inh_ms = 10.f;
  c->tau_adapt_ms = 200.f;
  c->adapt_inc_pa = 15.f;
  c->bias_pa = 0.f;
  c->drive_kind = NG_DRIVE_CONDUCTANCE;
  c->drive_p = 0.02f;
  c->drive_ns = 4.f;
  c->storage = 0;
  c->launch = 0;
  c->part_rank = 0;
  c->part_world = 0;
  // BiologyConfig learning defaults (biology.py:31-34); off unless asked for.
  c->plasticity = 0;
  c->stdp_rate = .005f;
  c->inhibitory_rate = .002f;
  c->target_hz = 5.f;
  c->scaling_tau_ms = 100000.f;
}

void *ng_net_create(const ng_net_config *cfg) {
  return guarded_ptr([&]() -> void * {
    if (!cfg) throw std::invalid_argument("Null network config");
    if (cfg->part_world > 1) throw std::invalid_argument("Use ng_net_create_partitioned for part_world > 1");
    // Fixed fan-in fp16 networks in CSR storage draw their synapses on the device.
    if (cfg->topology == NG_TOPO_FIXED_FANIN && cfg->weight_kind == NG_W_HALFNORMAL_F16 && cfg->storage == 0)
      return new Network(*cfg, nullptr, DeviceFanin{});
    std::unique_ptr<Topology> t(make_topology(*cfg));
    return new Network(*t);
  });
}

void *ng_net_create_edges(const ng_net_config *cfg, int64_t n_syn, const int32_t *pre, const int32_t *post,
                          const int32_t *delay, const float *weight) {
  return guarded_ptr([&]() -> void * {
    if (!cfg) throw std::invalid_argument("Null network config");
    std::unique_ptr<Topology> t(make_topology_edges(*cfg, n_syn, pre, post, delay, weight));
    return new Network(*t);
  });
}

void *ng_net_create_topology(const void *topology) {
  return guarded_ptr([&]() -> void * {
    if (!topology) throw std::invalid_argument("Null topology");
    return new Network(*static_cast<const Topology *>(topology));
  });
}

void *ng_net_create_partitioned(const ng_net_config *cfg, const void *nccl_id) {
  return guarded_ptr([&]() -> void * {
    if (!cfg) throw std::invalid_argument("Null network config");
    if (cfg->part_world < 2) throw std::invalid_argument("ng_net_create_partitioned needs part_world >= 2");
    if (!nccl_id) throw std::invalid_argument("Null NCCL unique id");
    // Fixed fan-in fp16 networks (the large ones) draw their synapses on the device.
    if (cfg->topology == NG_TOPO_FIXED_FANIN && cfg->weight_kind == NG_W_HALFNORMAL_F16)
      return new Network(*cfg, nccl_id, DeviceFanin{});
    std::unique_ptr<Topology> t(make_topology(*cfg));
    return new Network(*t, nccl_id);
  });
}

int ng_nccl_unique_id(void *id) {
  return guarded([&] {
    if (!id) throw std::invalid_argument("Null output");
    ncclUniqueId u;
    nccl_check(nccl().GetUniqueId(&u), "ncclGetUniqueId");
    std::memcpy(id, &u, sizeof u);
  });
}

void *ng_topology_create(const ng_net_config *cfg) {
  return guarded_ptr([&]() -> void * {
    if (!cfg) throw std::invalid_argument("Null network config");
    return make_topology(*cfg);
  });
}

void ng_topology_destroy(void *topology) { delete static_cast<Topology *>(topology); }

int64_t ng_topology_synapses(const void *topology) {
  return topology ? static_cast<const Topology *>(topology)->synapses() : -1;
}

int ng_topology_export(const void *topology, int32_t *pre, int32_t *post, int32_t *delay, float *weight) {
  return guarded([&] {
    if (!topology) throw std::invalid_argument("Null topology");
    static_cast<const Topology *>(topology)->export_edges(pre, post, delay, weight);
  });
}

void ng_net_destroy(void *net) { delete static_cast<Network *>(net); }

int64_t ng_net_synapses(void *net) { return net ? static_cast<Network *>(net)->synapses() : -1; }

int ng_net_launch_kind(void *net) {
  if (!net) return -1;
  const Network &w = *static_cast<Network *>(net);
  if (w.resident()) return w.resident_plan().pipe ? 4 : 3;
  return w.split() ? 2 : 1;
}

int ng_net_plasticity_state(void *net, float *pre_trace, float *potential_trace, float *coactivity, float *usage,
                            float *post_trace, float *rate) {
  return guarded([&] {
    if (!net) throw std::invalid_argument("Null network");
    auto &n = *static_cast<Network *>(net);
    std::lock_guard<std::mutex> lock(n.mutex);
    n.plasticity_state(pre_trace, potential_trace, coactivity, usage, post_trace, rate);
  });
}

int ng_net_exchange_kind(void *net) {
  if (!net) return -1;
  const Network &w = *static_cast<Network *>(net);
  return w.exchange_kind();
}

int ng_net_export(void *net, int32_t *pre, int32_t *post, int32_t *delay, float *weight) {
  return guarded([&] {
    if (!net) throw std::invalid_argument("Null network");
    auto &n = *static_cast<Network *>(net);
    std::lock_guard<std::mutex> lock(n.mutex);
    n.export_edges(pre, post, delay, weight);
  });
}

int ng_net_set_state(void *net, const float *v, const float *adapt, const float *g_exc, const float *g_inh,
                     const int32_t *refractory, const int32_t *ring, int64_t tick) {
  return guarded([&] {
    if (!net) throw std::invalid_argument("Null network");
    auto &n = *static_cast<Network *>(net);
    std::lock_guard<std::mutex> lock(n.mutex);
    n.set_state(v, adapt, g_exc, g_inh, refractory, ring, tick);
  });
}

int ng_net_get_state(void *net, float *v, float *adapt, float *g_exc, float *g_inh, int32_t *refractory,
                     int32_t *ring, int64_t *tick) {
  return guarded([&] {
    if (!net) throw std::invalid_argument("Null network");
    auto &n = *static_cast<Network *>(net);
    std::lock_guard<std::mutex> lock(n.mutex);
    n.get_state(v, adapt, g_exc, g_inh, refractory, ring, tick);
  });
}

int ng_net_run(void *net, int ticks, uint32_t *spikes, int64_t *counts) {
  return guarded([&] {
    if (!net) throw std::invalid_argument("Null network");
    if (ticks < 0) throw std::invalid_argument("ticks must be non-negative");
    auto &n = *static_cast<Network *>(net);
    std::lock_guard<std::mutex> lock(n.mutex);
    n.run_host(ticks, spikes, counts);
  });
}

int ng_net_stats(void *net, int64_t *totals) {
  return guarded([&] {
    if (!net || !totals) throw std::invalid_argument("Null network or output");
    auto &n = *static_cast<Network *>(net);
    std::lock_guard<std::mutex> lock(n.mutex);
    n.stats(totals);
  });
}

int ng_net_run_device(void *net, int ticks, uint32_t *d_spikes, int64_t *d_counts, void *stream) {
  return guarded([&] {
    if (!net) throw std::invalid_argument("Null network");
    auto &n = *static_cast<Network *>(net);
    std::lock_guard<std::mutex> lock(n.mutex);
    NGB_CUDA(cudaSetDevice(n.device));
    n.enqueue(ticks, d_spikes, reinterpret_cast<unsigned long long *>(d_counts),
              stream ? static_cast<cudaStream_t>(stream) : n.stream);
  });
}

} // extern "C"
