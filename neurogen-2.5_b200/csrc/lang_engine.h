// Device-resident language model: dims, weights in HBM, scratch, and the
// launch sequence of one token / one advance for a batch of sessions.
#pragma once
#include "common.h"
#include "engine/NeuralEngine.h"
#include "lang_kernels.h"

#include <string>
#include <vector>

namespace ngb {

constexpr int kVocab = 264; // bytes + 8 control tokens (neurogen/language/model.py:16-17)

struct LangDims {
  LangDims(const neurogen::cortical::EngineConfig &cfg, const neurogen::cortical::CorticalColumnV2 &col);
  int c, w, R, T, idle;
  int n;                 // units per region (c*64)
  int n_in, n_fb, n_out; // 12, 29, 50 per column
  long RS;               // floats per region state block: 5n + w
  long S;                // floats per session state: R * RS
};

struct RegionWeights {
  DeviceBuffer rec;                     // [c][64][64], transformed
  DeviceBuffer in_wp, in_b;             // panels of [c*n_in][w], bias
  DeviceBuffer fb_wp;                   // panels of [c*n_fb][w]
  DeviceBuffer out_wp, out_b;           // panels of [w][c*n_out*2], bias
  DeviceBuffer in_wr, fb_wr, out_wr;    // the same three row-major (small-batch kernel)
  // tf32 hi / lo splits of the three row-major matrices (tensor-core projections only)
  DeviceBuffer in_hi, in_lo, fb_hi, fb_lo, out_hi, out_lo;
  DeviceBuffer norm_w, norm_b, decay;   // [w]
};

// Device working memory one token step / advance needs, as raw pointers
// (sizes for B sessions: h, hraw [B][w]; vin [B][c*n_in]; fb [R][B][c*n_fb];
// tr [B][n]; feat [B][c*n_out*2]; cnt int [B][1+idle][R]).
struct ScratchView {
  float *h, *hraw, *vin, *fb, *tr, *feat;
  int *cnt;
  float *h_hi = nullptr, *h_lo = nullptr; // tf32 split of h for the tensor-core readout, or null
  float *x_hi = nullptr, *x_lo = nullptr; // [B][max K] tf32 split of a projection's input, or null
};

// Per-call device workspace for `capacity` sessions.
struct Scratch {
  int capacity = 0;
  DeviceBuffer h, hraw, vin, fb, tr, feat, cnt, tokens, inputs, state, logits, hidden, act, h_hi, h_lo, x_hi, x_lo;
  void ensure(const LangDims &d, int batch, bool tc_proj);
  ScratchView view() const {
    return {h.as<float>(),   hraw.as<float>(), vin.as<float>(),  fb.as<float>(),  tr.as<float>(),
            feat.as<float>(), cnt.as<int>(),    h_hi.as<float>(), h_lo.as<float>(), x_hi.as<float>(),
            x_lo.as<float>()};
  }
};

class DeviceModel {
public:
  DeviceModel(const neurogen::cortical::EngineConfig &cfg,
              const neurogen::cortical::CorticalColumnV2 &col, const float *packed);
  ~DeviceModel();
  DeviceModel(const DeviceModel &) = delete;
  DeviceModel &operator=(const DeviceModel &) = delete;

  // Enqueue `advances` advances of B sessions whose state [B][S] is on the
  // device and is updated in place.  The first advance reads the embedding
  // rows d_tokens (token step) or the inputs d_inputs [B][w]; it is idle when
  // first_idle is set.  Outputs may be null.
  void enqueue(int B, const int *d_tokens, const float *d_inputs, bool first_idle, int advances,
               float *d_state, float *d_logits, float *d_hidden, float *d_act, Scratch &sc,
               cudaStream_t st) const {
    enqueue_view(B, d_tokens, d_inputs, first_idle, advances, d_state, d_logits, d_hidden, d_act, sc.view(), st);
  }
  // The same launch sequence on caller-provided working memory.
  void enqueue_view(int B, const int *d_tokens, const float *d_inputs, bool first_idle, int advances,
                    float *d_state, float *d_logits, float *d_hidden, float *d_act, const ScratchView &sc,
                    cudaStream_t st) const;

  LangDims dims;
  int device = 0;
  std::string label;
  cudaStream_t stream = nullptr;
  UnitTables tables;
  // Device copies of the host-libm correction tables (math_tables.h).
  DeviceBuffer sig_start, sig_entries, sig_map, sig_skip, sig_neg_start, sig_neg_entries, sig_neg_map, sig_neg_skip,
      tanh_start, tanh_entries, tanh_map, tanh_skip;
  libm_match::MathTable sig_tab, sig_neg_tab, tanh_tab;
  DeviceBuffer emb, head_wp, head_b, head_wr;
  DeviceBuffer head_hi, head_lo; // tf32 split of head_wr for the tensor-core readout
  // Batched projections on the tensor cores too (NEUROGEN_PROJECTION=tc at
  // model load); the exact sequential projections otherwise.
  bool tc_proj = false;
  std::vector<RegionWeights> regions;
  Scratch host_scratch; // used by the host-buffer entry points (under the engine mutex)
  // Error word of the tensor-core readout (pinned, mapped into the device):
  // nonzero after one of its bounded waits timed out.
  int *readout_err = nullptr, *readout_err_dev = nullptr;
  // Throws when a kernel reported an error; call after synchronising.
  void check_device_errors() const;
};

} // namespace ngb
