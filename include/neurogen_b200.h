/*
 * neurogen_b200.h -- C ABI of libneurogen_native.so, the B200 (sm_100a) engine.
 *
 * Plain C: no CUDA, PyTorch or C++ types cross this boundary.  Every entry
 * point returns 0 / a non-null handle on success and -1 / NULL on failure; the
 * failure text is available from ng_error() (thread-local, valid until the
 * next call on the same thread).  There is no silent fallback: when no usable
 * sm_100 device is present, creation fails with an explanatory error.
 *
 * Part 1 is the reference's own ABI, same names, argument meaning and error
 * behaviour, so existing ctypes/cgo bindings load this library unchanged.
 * Parts 2-4 are additions (batched sessions, device-resident session pools and
 * the isolated spiking-network tick engine); they follow the same conventions.
 */
#ifndef NEUROGEN_B200_H
#define NEUROGEN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------ */
/* Part 1: reference-compatible language-core ABI.                           */
/* ------------------------------------------------------------------------ */

/* Replaces ng_create, include/engine/NeuralEngine.h:35-36 (impl
 * src/native/NeuralEngine.cpp:208-218).  `weights` is the packed fp32 stream in
 * the order of neurogen/language/native.py:46-52; `backend` must be "cuda"
 * (or NULL, which means "cuda" here).  Weights are copied to the device once. */
void *ng_create(int columns, int width, int regions, int ticks, int idle_steps,
                const float *weights, size_t count, const char *backend);

/* Replaces ng_destroy, NeuralEngine.h:37 (NeuralEngine.cpp:219). */
void ng_destroy(void *engine);

/* Replaces ng_error, NeuralEngine.h:38 (NeuralEngine.cpp:220). */
const char *ng_error(void);

/* Replaces ng_backend, NeuralEngine.h:39 (NeuralEngine.cpp:221-226). */
const char *ng_backend(void *engine);

/* Replaces ng_step, NeuralEngine.h:40-41 (NeuralEngine.cpp:227-246).  One token
 * for one session; caller-owned host state in, next state out. */
int ng_step(void *engine, int token, const float *state, size_t state_count,
            float *next_state, float *logits, float *hidden, float *activity);

/* Replaces ng_advance, NeuralEngine.h:42-44 (NeuralEngine.cpp:247-267). */
int ng_advance(void *engine, const float *input, const float *state,
               size_t state_count, int idle, float *next_state, float *hidden,
               float *activity);

/* ------------------------------------------------------------------------ */
/* Part 2: batched sessions on host buffers.                                 */
/* ------------------------------------------------------------------------ */

/* Sizes of an engine (reference NeuralEngine::state_size / parameter_count,
 * src/native/NeuralEngine.cpp:133-139). */
size_t ng_state_size(void *engine);
size_t ng_parameter_count(int columns, int width, int regions);

/* `batch` independent sessions in one call.  Replaces the per-item Python
 * loop of neurogen/language/native.py:128-137.  state/next_state are
 * [batch, state_count] row-major; logits [batch, 264]; hidden [batch, width];
 * activity [batch].  state and next_state may alias. */
int ng_step_batch(void *engine, const int *tokens, int batch, const float *state,
                  size_t state_count, float *next_state, float *logits,
                  float *hidden, float *activity);

/* inputs [batch, width]. */
int ng_advance_batch(void *engine, const float *inputs, int batch,
                     const float *state, size_t state_count, int idle,
                     float *next_state, float *hidden, float *activity);

/* Same as ng_step, but it allocates no device memory of its own: the state
 * staging, the activations between kernels and the outputs live in a fixed
 * 1 MiB array compiled into this library (every GPU that loads the library
 * holds it until exit).  No counterpart in the reference.  For callers that
 * cannot have a step allocate -- a fixed device-memory budget, or a streaming
 * loop where a cudaMalloc could block on the driver's allocation lock and
 * synchronise the device.  Models whose step needs more than 262,144 floats
 * of working memory are rejected with an error (BC-250 needs ~57k).  The
 * first call on a device looks the array up and loads the kernels; make it
 * before any stream capture.  Calls share the array: this process serialises
 * them per device, and calls that overlap on the GPU from other means would
 * race.  The array's address is looked up once per device and kept: the
 * library assumes the device's primary context lives as long as the process
 * (after a cudaDeviceReset, create the engine anew in a new process). */
int ng_step_static(void *engine, int token, const float *state,
                   size_t state_count, float *next_state, float *logits,
                   float *hidden, float *activity);

/* The input sigmoid 1/(1 + expf(-x)) and the feedback tanhf exactly as the
 * tick kernels evaluate them on the device, for n inputs (host buffers;
 * either output may be NULL).  They equal the host C library's values, which
 * the reference CPU engine uses (NeuralEngine.cpp:9,84-85); this entry point
 * exists to check that.  No reference counterpart. */
int ng_math_eval(const float *x, size_t n, float *tanh_out, float *sigmoid_out);

/* ------------------------------------------------------------------------ */
/* Part 3: device-resident session pools (state stays in HBM between calls). */
/* ------------------------------------------------------------------------ */

/* A pool of `batch` sessions whose state lives on the engine's device,
 * zero-initialised (the reference model's initial state, model.py:68-70). */
void *ng_pool_create(void *engine, int batch);
void ng_pool_destroy(void *pool);
/* Copy all session states in/out, host layout [batch, state_size]. */
int ng_pool_load(void *pool, const float *state);
int ng_pool_store(void *pool, float *state);
/* One token per session: tokens [batch] (host), logits [batch, 264] (host,
 * may be NULL), hidden [batch, width] and activity [batch] may be NULL. */
int ng_pool_step(void *pool, const int *tokens, float *logits, float *hidden,
                 float *activity);
/* Same with device pointers on a caller stream (cudaStream_t as void*; NULL =
 * the engine's stream).  Enqueues only; does not synchronise. */
int ng_pool_step_device(void *pool, const int *d_tokens, float *d_logits,
                        void *stream);
/* Device pointer to the pool's state [batch, state_size]. */
float *ng_pool_device_state(void *pool);

/* ------------------------------------------------------------------------ */
/* Part 4: isolated-tick spiking network (conductance ALIF + delay ring).    */
/* ------------------------------------------------------------------------ */

/* Topology kinds of a generated network. */
enum {
  NG_TOPO_ERDOS_RENYI = 0, /* each ordered pair (pre != post) with prob p_connect */
  NG_TOPO_FIXED_FANIN = 1, /* each post draws exactly `fanin` uniform pres      */
  NG_TOPO_BSR16 = 2        /* 16x16 blocks: per block-row `bsr_blocks` uniform
                              block-columns, each with exactly `bsr_fill` of its
                              256 entries non-zero                               */
};
/* Weight distributions (magnitudes; inhibitory presynaptic rows negated). */
enum {
  NG_W_LOGNORMAL_F32 = 0, /* exp(N(w_mu, w_sigma)), stored fp32 */
  NG_W_HALFNORMAL_F16 = 1 /* |N(0, w_sigma)|, stored fp16        */
};
/* External drive. */
enum {
  NG_DRIVE_CONDUCTANCE = 0, /* Bernoulli(drive_p) event adds drive_ns to g_E   */
  NG_DRIVE_IMPOSED = 1      /* each neuron spikes with Bernoulli(drive_p); the
                               threshold is not applied                        */
};

typedef struct {
  /* topology */
  int32_t n;          /* neurons */
  int32_t n_exc;      /* the first n_exc neurons are excitatory */
  int32_t topology;   /* NG_TOPO_* */
  float p_connect;    /* Erdos-Renyi probability */
  int32_t fanin;      /* fixed fan-in */
  int32_t bsr_blocks; /* BSR: block-columns per block-row */
  int32_t bsr_fill;   /* BSR: non-zeros per 16x16 block */
  int32_t weight_kind; /* NG_W_* */
  float w_mu, w_sigma;
  int32_t delay_min, delay_max; /* ticks, 1 <= min <= max <= 15 */
  uint64_t seed;
  /* dynamics (biology.py units: ms, mV, pA, pF, nS) */
  float dt_ms;
  float cap_exc_pf, cap_inh_pf; /* 200, 100 */
  float g_leak_ns;              /* 10 */
  float e_leak_mv, e_inh_mv;    /* -65, -80 (E_exc is 0) */
  float v_thresh_mv, v_reset_mv; /* -50, -65 */
  float t_ref_ms;               /* 2 */
  float tau_exc_ms, tau_inh_ms, tau_adapt_ms; /* 5, 10, 200 */
  float adapt_inc_pa;           /* 15 (excitatory cells only) */
  float bias_pa;                /* constant injected current */
  int32_t drive_kind;           /* NG_DRIVE_* */
  float drive_p;                /* Bernoulli probability per neuron per tick */
  float drive_ns;               /* conductance added per drive event */
  int32_t storage;              /* 0 = CSR push, 1 = BSR push (BSR16 topology) */
  int32_t launch;               /* 0 = auto, 1 = one fused launch per tick,
                                   2 = split membrane / push launches,
                                   3 = resident: one persistent launch runs many
                                   ticks with neuron state and delay ring in
                                   shared memory (unpartitioned; its per-owner
                                   event blocks are built from either storage).
                                   Auto picks 3 when the network fits, else 1
                                   below 65,536 neurons, else 2.                */
  int32_t part_rank, part_world; /* neuron row-partition: this rank owns neurons
                                   [rank*n/world, (rank+1)*n/world); 0/1 = whole */
  /* Learning (biology.py:182-218): pair STDP with soft bounds on E contacts, the
   * inhibitory rule on I->E contacts, multiplicative synaptic scaling toward
   * target_hz, weights clipped to [0.01, 4] (E) / [0.01, 12] (I); the tick's
   * emissions carry the learned weights.  Needs fp32 weights, CSR storage and an
   * unpartitioned network; runs the split launch shape, one tick after another. */
  int32_t plasticity;           /* 0 frozen synapses (default), 1 learn every tick */
  float stdp_rate;              /* .005 */
  float inhibitory_rate;        /* .002 */
  float target_hz;              /* 5 */
  float scaling_tau_ms;         /* 100000 */
  int32_t reserved[3];
} ng_net_config;

/* Fill `cfg` with the biology.py defaults (BiologyConfig, biology.py:19-77;
 * membrane constants biology.py:160-170) and a small Erdos-Renyi topology. */
void ng_net_default_config(ng_net_config *cfg);

/* Generate the network described by `cfg` (deterministic in cfg->seed) and
 * upload it to the current CUDA device.  Fixed fan-in networks with fp16
 * weights in CSR storage are drawn on the device (same draws as
 * ng_topology_create; the order of synapses inside a row may differ, spikes
 * and state do not).  Returns NULL on error. */
void *ng_net_create(const ng_net_config *cfg);

/* Build a network from caller arrays instead of generating one: synapse list
 * (pre[i] -> post[i], delay[i] ticks, weight[i] nS, negative = inhibitory).
 * Weights must be multiples of 2^-24 nS (the ring's fixed-point unit). */
void *ng_net_create_edges(const ng_net_config *cfg, int64_t n_syn,
                          const int32_t *pre, const int32_t *post,
                          const int32_t *delay, const float *weight);
void ng_net_destroy(void *net);

/* Neuron-partitioned network over `part_world` GPUs (one process per GPU):
 * this rank owns the neurons [rank*n/world, (rank+1)*n/world) -- their state,
 * their delay-ring slots and every synapse that ends on them -- and the ranks
 * all-gather the per-tick spike bitmask (n/8 bytes in total) with NCCL over
 * NVLink.  Every rank calls this collectively with the same cfg (part_rank set
 * to its own rank) and the same 128-byte NCCL unique id from
 * ng_nccl_unique_id on one rank.  n must be a multiple of 32 * world; CSR
 * storage only.  Spikes and state equal those of the unpartitioned network. */
void *ng_net_create_partitioned(const ng_net_config *cfg, const void *nccl_id);
/* Fills `id` (128 bytes) with a fresh NCCL unique id. */
int ng_nccl_unique_id(void *id);

/* Host-only topology: generate the synapses of `cfg` without a GPU (the same
 * synapses ng_net_create would build), export them, or build a device network
 * from them.  Lets a CPU checker and the GPU share one generated network. */
void *ng_topology_create(const ng_net_config *cfg);
void ng_topology_destroy(void *topology);
int64_t ng_topology_synapses(const void *topology);
int ng_topology_export(const void *topology, int32_t *pre, int32_t *post,
                       int32_t *delay, float *weight);
void *ng_net_create_topology(const void *topology);

/* Synapse count, and export of the (generated) synapse list in the order
 * pre-major (arrays sized ng_net_synapses).  For a partitioned network: this
 * rank's synapses, with global neuron indices. */
int64_t ng_net_synapses(void *net);

/* Launch shape the network runs with: 1 fused, 2 split, 3 resident with the
 * serial tick, 4 resident with the pipelined tick; -1 on a null handle.  No counterpart in the reference (its isolated-tick network is
 * biology.py's NumPy loop). */
int ng_net_launch_kind(void *net);

/* How a partitioned network's ranks exchange each tick's spikes: 0 not
 * partitioned, 1 NCCL all-gather, 2 one-sided stores into every rank's buffers
 * over NVLink with tick-stamped flags (the default when every rank can map the
 * others' memory; NEUROGEN_PEER_EXCHANGE=0 selects NCCL); -1 on a null handle.
 * No counterpart in the reference. */
int ng_net_exchange_kind(void *net);
int ng_net_export(void *net, int32_t *pre, int32_t *post, int32_t *delay,
                  float *weight);

/* State: v, adapt, g_exc, g_inh (fp32 [n] each), refractory ticks (int32 [n]),
 * delay ring (int32 [16][n][2]) and the tick counter.  NULL pointers skip.
 * For a partitioned network n is this rank's neuron count, and ng_net_set_state
 * is collective (every rank calls it, with the same tick). */
int ng_net_set_state(void *net, const float *v, const float *adapt,
                     const float *g_exc, const float *g_inh,
                     const int32_t *refractory, const int32_t *ring,
                     int64_t tick);
int ng_net_get_state(void *net, float *v, float *adapt, float *g_exc,
                     float *g_inh, int32_t *refractory, int32_t *ring,
                     int64_t *tick);

/* Advance `ticks` ticks.  spikes (host, may be NULL): [ticks][ceil(n/32)]
 * uint32 bitmask words, bit (i % 32) of word i/32 = neuron i spiked (for a
 * partitioned network: the whole network's bitmask, on every rank).
 * counts (host, may be NULL): [ticks] spikes per tick. */
int ng_net_run(void *net, int ticks, uint32_t *spikes, int64_t *counts);

/* Running totals since creation: totals[0] = spikes, totals[1] = synaptic
 * events delivered (host array of 2).  Synchronises the network's stream. */
int ng_net_stats(void *net, int64_t *totals);

/* Learning state of a plasticity network (cfg.plasticity = 1): per contact, in
 * the order of ng_net_export, the pre trace, potential trace, coactivity and
 * usage (Hz); per neuron the postsynaptic trace and the rate (Hz), as
 * biology.py's BiologicalNetwork holds them.  The weights themselves come from
 * ng_net_export.  NULL pointers skip; -1 if the network does not learn.  No
 * counterpart in the reference's C ABI (its learning network is biology.py). */
int ng_net_plasticity_state(void *net, float *pre_trace, float *potential_trace,
                            float *coactivity, float *usage, float *post_trace,
                            float *rate);

/* Device-side run on a caller stream (NULL = the network's stream): no host
 * copies, no synchronisation.  d_spikes/d_counts may be NULL. */
int ng_net_run_device(void *net, int ticks, uint32_t *d_spikes,
                      int64_t *d_counts, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* NEUROGEN_B200_H */
