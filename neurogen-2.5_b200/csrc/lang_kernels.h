// Launch interface of the language-core kernels (lang_kernels.cu).  Plain
// structs of device pointers and sizes; the host engine (lang_engine.cpp)
// builds them.  All kernels reproduce the reference CPU engine's fp32
// arithmetic operation by operation (see lang_kernels.cu).
#pragma once
#include "libm_match.cuh"

#include <cuda_runtime.h>
#include <cstdint>

namespace ngb {

// Unit tables of a 64-unit column (derived from the laminar table,
// include/engine/ALIFNeuron.h): index of each unit in the input / feedback /
// output id lists, or -1, and a bitmask of excitatory units.
struct UnitTables {
  int8_t in_idx[64], fb_idx[64], out_idx[64];
  uint64_t exc_mask;
  int n_in, n_fb, n_out;
};

// y[b][m] = bias[m] + sum_{k=0..K-1, in order} W[m][k] * x[b][k]
//           (+ 0.25f * addv[b][m] when addv is set)
// W is stored in 32-row panels: W[m][k] at wp[(m/32)*K*32 + k*32 + m%32].
// Row b of x is x + (xidx ? xidx[b] : b) * ldx.
struct ProjArgs {
  const float *wp;
  const float *wr;   // the same weights row-major [M][K] (small-batch kernel), or null
  const float *bias; // [M] or null
  const float *x;
  const int *xidx; // optional row gather (embedding lookup)
  long ldx;
  float *y;
  long ldy;
  const float *addv; // optional 0.25 * addv epilogue
  long ldadd;
  int M, K, B;
};
void launch_projection(const ProjArgs &a, cudaStream_t s);
// Up to 4 independent projections (e.g. every region's feedback) in one launch.
struct ProjBatch {
  ProjArgs a[4];
  int count;
};
void launch_projections(const ProjBatch &pb, cudaStream_t s);

// Token readout y[b][v] = bias[v] + sum_k h[b][k] * w[v][k] on the tcgen05
// tensor cores (readout_tc.cu): split-tf32 operands, fp32 TMEM accumulators.
// Each operand comes as hi = x with the low 13 mantissa bits cleared and
// lo = x - hi (tf32_split / k_norm's split output).  Deterministic and within
// a few 1e-6 of the logit vector's scale of the sequential fp32 sum, but not
// bit-identical to it.  *err (device-visible, may be null) is set to 1 when a
// bounded wait in the kernel timed out.
struct ReadoutArgs {
  const float *h_hi, *h_lo; // [B] rows of K, row stride ldh
  long ldh;
  const float *w_hi, *w_lo; // [V][K] row-major
  const float *bias;        // [V] or null
  float *y;          // [B] rows of V, row stride ldy
  long ldy;
  int B, K, V;
  int *err;
  // Test switch: non-zero makes the launch give up before it issues any copy
  // or MMA, as a wait that ran out would (set by launch_readout_tc only).
  int stall_test;
  // Optional epilogue y[b][v] += 0.25f * addv[b * ldadd + v] (the output
  // projection's memory term), after the bias and the k sum.
  const float *addv;
  long ldadd;
};
// False when NEUROGEN_READOUT=simt is set (the sequential SIMT projection is
// then used at every batch size).
bool readout_tc_enabled();
// Shapes the kernel takes: B >= 2, K a multiple of 4, 16-byte aligned rows.
bool readout_tc_ok(const ReadoutArgs &a);
// Launches when readout_tc_ok(a); returns false (nothing launched) otherwise.
bool launch_readout_tc(const ReadoutArgs &a, cudaStream_t s);
// tf32 split of B rows of K floats (row b of x at x + (xidx ? xidx[b] : b) * ldx)
// into hi / lo [B][K], for a projection on the tensor cores.
void launch_tf32_split(const float *x, const int *xidx, long ldx, int K, int B, float *hi, float *lo,
                       cudaStream_t s);
// True when NEUROGEN_PROJECTION=tc: batched projections (B >= 2) run on the
// tensor cores as well (split-tf32, not bit-identical to the sequential sum).
bool projection_tc_enabled();
void configure_readout_tc();
const void *readout_tc_kernel();
// Per-device kernel attributes (dynamic shared memory); call once per device
// before launching, outside any stream capture.
void configure_lang_kernels();
// Forces every language-core kernel to be loaded on the current device now
// (under lazy module loading a first launch would otherwise load it).
void preload_lang_kernels();

// One synchronous recurrent ALIF tick of one region for B sessions
// (reference CPUBackend.cpp:20-42 with the input current assembled as in
// NeuralEngine.cpp:72-86).  State block of session b, this region:
// state + b*S + roff : [V n][trace n][adapt n][last n][memory w][counts n].
struct TickArgs {
  const float *rec; // [c][64][64] transformed recurrent weights
  float *state;
  long S, roff;
  int n, c, w, B;
  const float *tr_in; // previous trace, per session stride tr_in_ld
  long tr_in_ld;
  float *tr_out;
  long tr_out_ld;
  const float *vin; // input projection [B][c*n_in] or null (non-sensory)
  const float *fb;  // feedback projection [B][c*n_fb]
  float *feat;      // [B][c*n_out*2] written when non-null (last tick)
  int *spikes;      // spike counter per session, stride spikes_ld
  long spikes_ld;
  UnitTables tab;
  // Corrections that make the input sigmoid and feedback tanh equal the host
  // C library's (libm_match.cuh).
  libm_match::MathTable sig_tab, sig_neg_tab, tanh_tab;
};
void launch_tick(const TickArgs &a, cudaStream_t s);
// All `ticks` ticks of one region in one thread-block-cluster launch (trace
// read from and written back to the state; tr_in/tr_out unused).  Returns
// false, launching nothing, when the column count has no cluster shape.
bool launch_ticks_cluster(const TickArgs &a, int ticks, cudaStream_t s);

// Copy trace src (stride src_ld) -> dst (stride dst_ld), n floats per session.
void launch_copy_rows(const float *src, long src_ld, float *dst, long dst_ld,
                      int n, int B, cudaStream_t s);

// h = LayerNorm(hraw) * norm_w + norm_b (mean/variance in fp64), then
// memory = decay * memory + (1 - decay) * h  (NeuralEngine.cpp:96-108).
struct NormArgs {
  const float *hraw;
  long hraw_ld;
  float *h;
  long h_ld;
  float *h_hi, *h_lo; // optional tf32 split of h (same row stride): hi = h with the low
                      // 13 mantissa bits cleared, lo = h - hi; null to skip
  float *mem;
  long mem_ld;
  const float *norm_w, *norm_b, *decay;
  int w, B;
};
void launch_norm(const NormArgs &a, cudaStream_t s);

// activity[b] from integer spike counts [B][A][R]
// (PackedBackend.h:50-53, NeuralEngine.cpp:164-189).
void launch_activity(const int *counts, int A, int R, int n, int T, float *act,
                     int B, cudaStream_t s);

} // namespace ngb
