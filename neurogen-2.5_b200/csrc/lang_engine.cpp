// Host side of the language core: weight unpacking/transforms, device
// layouts, and the per-token launch sequence.  Public C++ types keep the
// reference's names (include/engine/*.h); the compute runs on the GPU with all
// weights resident in HBM, uploaded once at construction.
#include "engine/NeuralEngine.h"
#include "lang_engine.h"
#include "math_tables.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <stdexcept>

namespace neurogen::cortical {

// Unit tables from the laminar table: units are numbered layer by layer,
// excitatory cells first within a layer.  Input goes to layer-4 excitatory
// cells, feedback to layers 1, 5 and 6, and every excitatory cell is read out
// (reference CorticalColumnV2 constructor, src/native/NeuralEngine.cpp:16-31).
CorticalColumnV2::CorticalColumnV2(CorticalColumnConfig config) : config_(config) {
  for (const LayerParams &lp : layers) {
    const int cells = lp.excitatory + lp.inhibitory;
    for (int k = 0; k < cells; ++k) {
      const int unit = static_cast<int>(sign_.size());
      const bool excitatory = k < lp.excitatory;
      sign_.push_back(excitatory ? 1.f : -1.f);
      layer_.push_back(lp.layer);
      if (excitatory && lp.layer == 4) input_ids_.push_back(unit);
      if (lp.layer == 1 || lp.layer >= 5) feedback_ids_.push_back(unit);
      if (excitatory) output_ids_.push_back(unit);
    }
  }
}

// Packed parameters of one region, in stream order: recurrent c*64*64, input
// weights+bias, feedback weights, output weights+bias, norm weight, norm
// bias, memory decay (src/native/NeuralEngine.cpp:32-37, 57-64).
size_t CorticalColumnV2::parameter_count() const {
  const size_t c = config_.columns, w = config_.width;
  return c * 64 * 64 + c * input_ids_.size() * (w + 1) + c * feedback_ids_.size() * w +
         w * (c * output_ids_.size() * 2 + 1) + 3 * w;
}

} // namespace neurogen::cortical

namespace ngb {
using neurogen::cortical::CorticalColumnV2;
using neurogen::cortical::EngineConfig;

namespace {

float sigmoid_host(float x) { return 1.f / (1.f + std::exp(-x)); }

// 32-row panel layout used by the projection kernels:
// W[m][k] -> out[(m/32)*K*32 + k*32 + m%32], rows padded with zeros.
std::vector<float> to_panels(const float *W, size_t M, size_t K) {
  const size_t P = (M + 31) / 32;
  std::vector<float> out(P * K * 32, 0.f);
  for (size_t m = 0; m < M; ++m)
    for (size_t k = 0; k < K; ++k) out[(m / 32) * K * 32 + k * 32 + m % 32] = W[m * K + k];
  return out;
}

DeviceBuffer upload(const float *host, size_t count) {
  DeviceBuffer d(count * sizeof(float));
  NGB_CUDA(cudaMemcpy(d.as<float>(), host, count * sizeof(float), cudaMemcpyHostToDevice));
  return d;
}
DeviceBuffer upload(const std::vector<float> &v) { return upload(v.data(), v.size()); }

} // namespace

LangDims::LangDims(const EngineConfig &cfg, const CorticalColumnV2 &col)
    : c(cfg.columns), w(cfg.width), R(cfg.regions), T(cfg.ticks), idle(cfg.idle_steps) {
  n = c * 64;
  n_in = static_cast<int>(col.input_ids().size());
  n_fb = static_cast<int>(col.feedback_ids().size());
  n_out = static_cast<int>(col.output_ids().size());
  RS = 5L * n + w;
  S = static_cast<long>(R) * RS;
}

void Scratch::ensure(const LangDims &d, int batch, bool tc_proj) {
  if (batch <= capacity) return;
  const size_t B = batch;
  h.reset(B * d.w * 4);
  hraw.reset(B * d.w * 4);
  vin.reset(B * d.c * d.n_in * 4);
  fb.reset(size_t(d.R) * B * d.c * d.n_fb * 4);
  tr.reset(B * d.n * 4);
  feat.reset(B * d.c * d.n_out * 2 * 4);
  cnt.reset(B * (1 + d.idle) * d.R * sizeof(int));
  tokens.reset(B * sizeof(int));
  inputs.reset(B * d.w * 4);
  state.reset(B * d.S * 4);
  logits.reset(B * kVocab * 4);
  hidden.reset(B * d.w * 4);
  act.reset(B * 4);
  h_hi.reset(B * d.w * 4);
  h_lo.reset(B * d.w * 4);
  if (tc_proj) {
    const size_t kmax = std::max<size_t>(d.w, size_t(d.c) * d.n_out * 2);
    x_hi.reset(B * kmax * 4);
    x_lo.reset(B * kmax * 4);
  }
  capacity = batch;
}

DeviceModel::DeviceModel(const EngineConfig &cfg, const CorticalColumnV2 &col, const float *data)
    : dims(cfg, col) {
  device = require_sm100_device();
  label = device_label(device);
  configure_lang_kernels();
  const LangDims &d = dims;
  const size_t c = d.c, w = d.w;

  // Unit tables for the kernels.
  std::memset(&tables, 0, sizeof tables);
  std::fill(std::begin(tables.in_idx), std::end(tables.in_idx), int8_t(-1));
  std::fill(std::begin(tables.fb_idx), std::end(tables.fb_idx), int8_t(-1));
  std::fill(std::begin(tables.out_idx), std::end(tables.out_idx), int8_t(-1));
  for (int k = 0; k < d.n_in; ++k) tables.in_idx[col.input_ids()[k]] = int8_t(k);
  for (int k = 0; k < d.n_fb; ++k) tables.fb_idx[col.feedback_ids()[k]] = int8_t(k);
  for (int k = 0; k < d.n_out; ++k) tables.out_idx[col.output_ids()[k]] = int8_t(k);
  for (int u = 0; u < 64; ++u)
    if (col.sign()[u] > 0) tables.exc_mask |= 1ull << u;
  tables.n_in = d.n_in;
  tables.n_fb = d.n_fb;
  tables.n_out = d.n_out;

  // Host-libm corrections of the tick kernels' sigmoid and tanh (built once
  // per process, uploaded per model).
  auto upload_table = [](const HostMathTable &h, DeviceBuffer &start, DeviceBuffer &entries, DeviceBuffer &map, DeviceBuffer &skip) {
    start.reset(h.start.size() * 4);
    entries.reset(std::max<size_t>(h.entries.size(), 1) * 2);
    NGB_CUDA(cudaMemcpy(start.as<void>(), h.start.data(), h.start.size() * 4, cudaMemcpyHostToDevice));
    if (!h.entries.empty())
      NGB_CUDA(cudaMemcpy(entries.as<void>(), h.entries.data(), h.entries.size() * 2, cudaMemcpyHostToDevice));
    libm_match::MathTable t;
    t.start = start.as<uint32_t>();
    t.entries = entries.as<uint16_t>();
    t.lo = h.lo;
    t.hi = h.hi;
    t.shift = h.shift;
    t.steps = h.steps;
    skip.reset(h.skip.size() * 4);
    NGB_CUDA(cudaMemcpy(skip.as<void>(), h.skip.data(), h.skip.size() * 4, cudaMemcpyHostToDevice));
    t.skip = skip.as<float>();
    if (!h.map.empty()) {
      map.reset(h.map.size() * 4);
      NGB_CUDA(cudaMemcpy(map.as<void>(), h.map.data(), h.map.size() * 4, cudaMemcpyHostToDevice));
      t.map = map.as<uint32_t>();
      t.map_lo = h.map_lo;
      t.map_hi = h.map_hi;
    }
    return t;
  };
  sig_tab = upload_table(sigmoid_table(false), sig_start, sig_entries, sig_map, sig_skip);
  sig_neg_tab = upload_table(sigmoid_table(true), sig_neg_start, sig_neg_entries, sig_neg_map, sig_neg_skip);
  tanh_tab = upload_table(tanh_table(), tanh_start, tanh_entries, tanh_map, tanh_skip);

  // Recurrent connectivity gain [post][pre] (laminar rule, no autapses).
  const std::vector<float> rec_gain = col.recurrent_gain();

  // tf32 split of a row-major matrix: hi = x with the low 13 mantissa bits
  // cleared (a tf32 value), lo = x - hi (exact in fp32).
  auto split_upload = [](const float *x, size_t count, DeviceBuffer &hi_dev, DeviceBuffer &lo_dev) {
    std::vector<float> hi(count), lo(count);
    for (size_t i = 0; i < count; ++i) {
      uint32_t bits;
      std::memcpy(&bits, x + i, 4);
      bits &= 0xFFFFE000u;
      std::memcpy(&hi[i], &bits, 4);
      lo[i] = x[i] - hi[i];
    }
    hi_dev = upload(hi);
    lo_dev = upload(lo);
  };
  tc_proj = projection_tc_enabled();

  const float *p = data;
  auto take = [&](size_t count) {
    const float *start = p;
    p += count;
    return start;
  };
  emb = upload(take(size_t(kVocab) * w), size_t(kVocab) * w);
  regions.resize(d.R);
  for (int r = 0; r < d.R; ++r) {
    RegionWeights &g = regions[r];
    // softplus(raw) * mask * sign, evaluated with the host libm exactly as the
    // reference loader does (max(raw,0) + log1p(exp(-|raw|))).
    const float *raw = take(c * 4096);
    std::vector<float> rec(c * 4096);
    for (size_t col_i = 0; col_i < c; ++col_i)
      for (int k = 0; k < 4096; ++k) {
        const float x = raw[col_i * 4096 + k];
        const float gain = rec_gain[k];
        rec[col_i * 4096 + k] =
            gain != 0.f ? (std::max(x, 0.f) + std::log1p(std::exp(-std::abs(x)))) * gain : 0.f;
      }
    g.rec = upload(rec);
    const float *in_w = take(c * d.n_in * w);
    g.in_wp = upload(to_panels(in_w, c * d.n_in, w));
    g.in_wr = upload(in_w, c * d.n_in * w);
    if (tc_proj) split_upload(in_w, c * d.n_in * w, g.in_hi, g.in_lo);
    g.in_b = upload(take(c * d.n_in), c * d.n_in);
    const float *fb_w = take(c * d.n_fb * w);
    g.fb_wp = upload(to_panels(fb_w, c * d.n_fb, w));
    g.fb_wr = upload(fb_w, c * d.n_fb * w);
    if (tc_proj) split_upload(fb_w, c * d.n_fb * w, g.fb_hi, g.fb_lo);
    const float *out_w = take(w * c * d.n_out * 2);
    g.out_wp = upload(to_panels(out_w, w, c * d.n_out * 2));
    g.out_wr = upload(out_w, w * c * d.n_out * 2);
    if (tc_proj) split_upload(out_w, w * c * d.n_out * 2, g.out_hi, g.out_lo);
    g.out_b = upload(take(w), w);
    g.norm_w = upload(take(w), w);
    g.norm_b = upload(take(w), w);
    const float *dec = take(w);
    std::vector<float> decay(w);
    for (size_t i = 0; i < w; ++i) decay[i] = .5f + .499f * sigmoid_host(dec[i]);
    g.decay = upload(decay);
  }
  const float *head_w = take(size_t(kVocab) * w);
  head_wp = upload(to_panels(head_w, kVocab, w));
  head_wr = upload(head_w, size_t(kVocab) * w);
  split_upload(head_w, size_t(kVocab) * w, head_hi, head_lo);
  head_b = upload(take(kVocab), kVocab);
  NGB_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
  NGB_CUDA(cudaHostAlloc(reinterpret_cast<void **>(&readout_err), sizeof(int), cudaHostAllocMapped));
  *readout_err = 0;
  NGB_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void **>(&readout_err_dev), readout_err, 0));
}

DeviceModel::~DeviceModel() {
  if (stream) cudaStreamDestroy(stream);
  if (readout_err) cudaFreeHost(readout_err);
}

// The flag is cleared as it is reported: the timed-out launch's logits are
// lost, but the sessions' state does not depend on the readout, so the next
// step on this engine runs normally.
void DeviceModel::check_device_errors() const {
  if (readout_err && *reinterpret_cast<volatile int *>(readout_err)) {
    *reinterpret_cast<volatile int *>(readout_err) = 0;
    throw std::runtime_error("Readout kernel timed out waiting for its tensor-core pipeline");
  }
}

void DeviceModel::enqueue_view(int B, const int *d_tokens, const float *d_inputs, bool first_idle,
                               int advances, float *d_state, float *d_logits, float *d_hidden,
                               float *d_act, const ScratchView &sc, cudaStream_t st) const {
  const LangDims &d = dims;
  const int A = advances;
  NGB_CUDA(cudaMemsetAsync(sc.cnt, 0, size_t(B) * A * d.R * sizeof(int), st));
  const int Min = d.c * d.n_in, Mfb = d.c * d.n_fb, Kout = d.c * d.n_out * 2;
  // Readout on the tensor cores when there is more than one session and the
  // split hidden state has somewhere to go; the sequential SIMT projection
  // otherwise.  The last LayerNorm writes the split.
  const ReadoutArgs ra{sc.h_hi, sc.h_lo, d.w, head_hi.as<float>(), head_lo.as<float>(), head_b.as<float>(),
                       d_logits, kVocab, B, d.w, kVocab, readout_err_dev};
  const bool tc_readout = d_logits && readout_tc_ok(ra);
  // A projection on the tensor cores (NEUROGEN_PROJECTION=tc, B >= 2): its
  // input split into tf32 hi / lo, then the readout kernel with the
  // projection's weights; the exact sequential kernel otherwise.
  const bool tc_proj_here = tc_proj && B >= 2 && sc.x_hi && sc.x_lo;
  auto project = [&](const ProjArgs &pa, const DeviceBuffer &w_hi, const DeviceBuffer &w_lo) {
    if (tc_proj_here) {
      launch_tf32_split(pa.x, pa.xidx, pa.ldx, pa.K, B, sc.x_hi, sc.x_lo, st);
      ReadoutArgs a{sc.x_hi, sc.x_lo, pa.K, w_hi.as<float>(), w_lo.as<float>(), pa.bias, pa.y, pa.ldy,
                    B, pa.K, pa.M, readout_err_dev};
      a.addv = pa.addv;
      a.ldadd = pa.ldadd;
      if (launch_readout_tc(a, st)) return;
    }
    launch_projection(pa, st);
  };
  for (int adv = 0; adv < A; ++adv) {
    const bool idle = adv > 0 || first_idle;
    // Feedback projections of every region read only that region's memory,
    // which the region updates after it has used them, so all regions'
    // feedback for this advance can be computed up front.
    for (int r0 = 0; r0 < d.R; r0 += 4) {
      ProjBatch fb{};
      fb.count = std::min(4, d.R - r0);
      for (int z = 0; z < fb.count; ++z) {
        const int r = r0 + z;
        ProjArgs &fa = fb.a[z];
        fa.wp = regions[r].fb_wp.as<float>();
        fa.wr = regions[r].fb_wr.as<float>();
        fa.x = d_state + r * d.RS + 4L * d.n;
        fa.ldx = d.S;
        fa.y = sc.fb + size_t(r) * B * Mfb;
        fa.ldy = Mfb;
        fa.M = Mfb;
        fa.K = d.w;
        fa.B = B;
      }
      if (tc_proj_here) {
        for (int z = 0; z < fb.count; ++z) project(fb.a[z], regions[r0 + z].fb_hi, regions[r0 + z].fb_lo);
      } else {
        launch_projections(fb, st);
      }
    }
    for (int r = 0; r < d.R; ++r) {
      const RegionWeights &g = regions[r];
      const bool sensory = !idle || r > 0;
      const long roff = r * d.RS;
      if (sensory) {
        ProjArgs ia{};
        ia.wp = g.in_wp.as<float>();
        ia.wr = g.in_wr.as<float>();
        ia.bias = g.in_b.as<float>();
        if (r == 0) {
          ia.x = d_tokens ? emb.as<float>() : d_inputs;
          ia.xidx = d_tokens;
        } else {
          ia.x = sc.h;
        }
        ia.ldx = d.w;
        ia.y = sc.vin;
        ia.ldy = Min;
        ia.M = Min;
        ia.K = d.w;
        ia.B = B;
        project(ia, g.in_hi, g.in_lo);
      }
      TickArgs ta{};
      ta.rec = g.rec.as<float>();
      ta.state = d_state;
      ta.S = d.S;
      ta.roff = roff;
      ta.n = d.n;
      ta.c = d.c;
      ta.w = d.w;
      ta.B = B;
      ta.vin = sensory ? sc.vin : nullptr;
      ta.fb = sc.fb + size_t(r) * B * Mfb;
      ta.spikes = sc.cnt + adv * d.R + r;
      ta.spikes_ld = long(A) * d.R;
      ta.tab = tables;
      ta.sig_tab = sig_tab;
      ta.sig_neg_tab = sig_neg_tab;
      ta.tanh_tab = tanh_tab;
      ta.feat = sc.feat;
      if (!launch_ticks_cluster(ta, d.T, st)) {
        // No cluster shape for this column count: one launch per tick with a
        // ping-pong trace buffer, then the trace back into the state.
        float *state_trace = d_state + roff + d.n;
        for (int t = 0; t < d.T; ++t) {
          ta.tr_in = t % 2 == 0 ? state_trace : sc.tr;
          ta.tr_in_ld = t % 2 == 0 ? d.S : d.n;
          ta.tr_out = t % 2 == 0 ? sc.tr : state_trace;
          ta.tr_out_ld = t % 2 == 0 ? d.n : d.S;
          ta.feat = t == d.T - 1 ? sc.feat : nullptr;
          launch_tick(ta, st);
        }
        if (d.T % 2 == 1) launch_copy_rows(sc.tr, d.n, state_trace, d.S, d.n, B, st);
      }
      ProjArgs oa{};
      oa.wp = g.out_wp.as<float>();
      oa.wr = g.out_wr.as<float>();
      oa.bias = g.out_b.as<float>();
      oa.x = sc.feat;
      oa.ldx = Kout;
      oa.y = sc.hraw;
      oa.ldy = d.w;
      oa.addv = d_state + roff + 4L * d.n; // memory before this region's update
      oa.ldadd = d.S;
      oa.M = d.w;
      oa.K = Kout;
      oa.B = B;
      project(oa, g.out_hi, g.out_lo);
      NormArgs na{};
      na.hraw = sc.hraw;
      na.hraw_ld = d.w;
      na.h = sc.h;
      na.h_ld = d.w;
      na.mem = d_state + roff + 4L * d.n;
      na.mem_ld = d.S;
      na.norm_w = g.norm_w.as<float>();
      na.norm_b = g.norm_b.as<float>();
      na.decay = g.decay.as<float>();
      na.w = d.w;
      na.B = B;
      if (tc_readout && adv == A - 1 && r == d.R - 1) {
        na.h_hi = sc.h_hi;
        na.h_lo = sc.h_lo;
      }
      launch_norm(na, st);
    }
  }
  if (d_logits) {
    if (!tc_readout || !launch_readout_tc(ra, st)) {
    ProjArgs ha{};
    ha.wp = head_wp.as<float>();
    ha.wr = head_wr.as<float>();
    ha.bias = head_b.as<float>();
    ha.x = sc.h;
    ha.ldx = d.w;
    ha.y = d_logits;
    ha.ldy = kVocab;
    ha.M = kVocab;
    ha.K = d.w;
    ha.B = B;
    launch_projection(ha, st);
    }
  }
  if (d_hidden)
    NGB_CUDA(cudaMemcpyAsync(d_hidden, sc.h, size_t(B) * d.w * 4, cudaMemcpyDeviceToDevice, st));
  if (d_act) launch_activity(sc.cnt, A, d.R, d.n, d.T, d_act, B, st);
  NGB_CUDA(cudaGetLastError());
}

} // namespace ngb

namespace neurogen::cortical {
using namespace ngb;

namespace {
void validate_dims(const EngineConfig &c) {
  if (c.columns < 1 || c.columns > 4096 || c.width < 1 || c.width > 16384 || c.regions < 1 ||
      c.regions > 128 || c.ticks < 1 || c.ticks > 10000 || c.idle_steps < 0 || c.idle_steps > 16)
    throw std::invalid_argument("Invalid native model dimensions");
}
bool all_finite(const float *p, size_t n) {
  for (size_t i = 0; i < n; ++i)
    if (!std::isfinite(p[i])) return false;
  return true;
}
} // namespace

NeuralEngine::NeuralEngine(EngineConfig c, const float *data, size_t count, const std::string &backend)
    : config(c) {
  validate_dims(c);
  if (!data || count != parameter_count())
    throw std::invalid_argument("Native weight count does not match architecture");
  if (!all_finite(data, count)) throw std::invalid_argument("Non-finite weights");
  if (backend != "cuda")
    throw std::invalid_argument("Native backend '" + backend +
                                "' unavailable; this library provides only 'cuda' "
                                "(B200, sm_100a) (no silent fallback)");
  CorticalColumnV2 column({c.columns, c.width, c.ticks});
  impl_ = std::make_unique<DeviceModel>(c, column, data);
}

NeuralEngine::~NeuralEngine() = default;

size_t NeuralEngine::parameter_count() const {
  CorticalColumnV2 column({config.columns, config.width, config.ticks});
  return 528ull * config.width + kVocab + size_t(config.regions) * column.parameter_count();
}

size_t NeuralEngine::state_size() const {
  return size_t(config.regions) * (5ull * config.columns * 64 + config.width);
}

std::string NeuralEngine::backend_name() const { return impl_->label; }

std::vector<ColumnState> NeuralEngine::unpack(const float *source) const {
  std::vector<ColumnState> out;
  const size_t n = size_t(config.columns) * 64, w = config.width;
  for (int r = 0; r < config.regions; ++r) {
    out.emplace_back(n, w);
    ColumnState &s = out.back();
    // Packed order per region: voltage, trace, adaptation, last_spikes,
    // memory, counts (src/native/NeuralEngine.cpp:145-151).
    for (std::vector<float> *f : {&s.neurons.voltage, &s.neurons.trace, &s.neurons.adaptation,
                                  &s.neurons.last_spikes, &s.memory, &s.neurons.counts}) {
      std::copy(source, source + f->size(), f->begin());
      source += f->size();
    }
  }
  return out;
}

void NeuralEngine::pack(const std::vector<ColumnState> &states, float *dest) const {
  for (const ColumnState &s : states)
    for (const std::vector<float> *f : {&s.neurons.voltage, &s.neurons.trace, &s.neurons.adaptation,
                                        &s.neurons.last_spikes, &s.memory, &s.neurons.counts}) {
      std::copy(f->begin(), f->end(), dest);
      dest += f->size();
    }
}

void NeuralEngine::step_batch(const int *tokens, int batch, const float *state, float *next_state,
                              float *logits, float *hidden, float *activity) {
  if (batch < 1) throw std::invalid_argument("Need at least one batch item");
  if (!tokens || !state || !next_state) throw std::invalid_argument("Null input/output");
  const size_t S = state_size();
  if (!all_finite(state, S * batch)) throw std::invalid_argument("Non-finite native state");
  for (int b = 0; b < batch; ++b)
    if (tokens[b] < 0 || tokens[b] >= kVocab) throw std::invalid_argument("Token must be in 0..263");
  DeviceModel &m = *impl_;
  NGB_CUDA(cudaSetDevice(m.device));
  Scratch &sc = m.host_scratch;
  sc.ensure(m.dims, batch, m.tc_proj);
  cudaStream_t st = m.stream;
  NGB_CUDA(cudaMemcpyAsync(sc.tokens.as<int>(), tokens, batch * sizeof(int), cudaMemcpyHostToDevice, st));
  NGB_CUDA(cudaMemcpyAsync(sc.state.as<float>(), state, S * batch * 4, cudaMemcpyHostToDevice, st));
  m.enqueue(batch, sc.tokens.as<int>(), nullptr, false, 1 + config.idle_steps, sc.state.as<float>(),
            sc.logits.as<float>(), sc.hidden.as<float>(), sc.act.as<float>(), sc, st);
  NGB_CUDA(cudaMemcpyAsync(next_state, sc.state.as<float>(), S * batch * 4, cudaMemcpyDeviceToHost, st));
  if (logits)
    NGB_CUDA(cudaMemcpyAsync(logits, sc.logits.as<float>(), size_t(batch) * kVocab * 4, cudaMemcpyDeviceToHost, st));
  if (hidden)
    NGB_CUDA(cudaMemcpyAsync(hidden, sc.hidden.as<float>(), size_t(batch) * config.width * 4, cudaMemcpyDeviceToHost, st));
  if (activity)
    NGB_CUDA(cudaMemcpyAsync(activity, sc.act.as<float>(), size_t(batch) * 4, cudaMemcpyDeviceToHost, st));
  NGB_CUDA(cudaStreamSynchronize(st));
  m.check_device_errors();
}

void NeuralEngine::advance_batch(const float *inputs, int batch, const float *state, bool idle,
                                 float *next_state, float *hidden, float *activity) {
  if (batch < 1) throw std::invalid_argument("Need at least one batch item");
  if (!inputs || !state || !next_state) throw std::invalid_argument("Null input/output");
  const size_t S = state_size();
  if (!all_finite(state, S * batch)) throw std::invalid_argument("Non-finite native state");
  if (!all_finite(inputs, size_t(config.width) * batch)) throw std::invalid_argument("Non-finite input");
  DeviceModel &m = *impl_;
  NGB_CUDA(cudaSetDevice(m.device));
  Scratch &sc = m.host_scratch;
  sc.ensure(m.dims, batch, m.tc_proj);
  cudaStream_t st = m.stream;
  NGB_CUDA(cudaMemcpyAsync(sc.inputs.as<float>(), inputs, size_t(batch) * config.width * 4, cudaMemcpyHostToDevice, st));
  NGB_CUDA(cudaMemcpyAsync(sc.state.as<float>(), state, S * batch * 4, cudaMemcpyHostToDevice, st));
  m.enqueue(batch, nullptr, sc.inputs.as<float>(), idle, 1, sc.state.as<float>(), nullptr,
            sc.hidden.as<float>(), sc.act.as<float>(), sc, st);
  NGB_CUDA(cudaMemcpyAsync(next_state, sc.state.as<float>(), S * batch * 4, cudaMemcpyDeviceToHost, st));
  if (hidden)
    NGB_CUDA(cudaMemcpyAsync(hidden, sc.hidden.as<float>(), size_t(batch) * config.width * 4, cudaMemcpyDeviceToHost, st));
  if (activity)
    NGB_CUDA(cudaMemcpyAsync(activity, sc.act.as<float>(), size_t(batch) * 4, cudaMemcpyDeviceToHost, st));
  NGB_CUDA(cudaStreamSynchronize(st));
  m.check_device_errors();
}

Vector NeuralEngine::step(int token, std::vector<ColumnState> &state, Vector &hidden, float &activity) {
  if (token < 0 || token >= kVocab) throw std::invalid_argument("Token must be in 0..263");
  std::vector<float> packed(state_size());
  pack(state, packed.data());
  Vector logits(kVocab);
  hidden.assign(config.width, 0.f);
  step_batch(&token, 1, packed.data(), packed.data(), logits.data(), hidden.data(), &activity);
  state = unpack(packed.data());
  return logits;
}

Vector NeuralEngine::advance(const Vector &input, std::vector<ColumnState> &state, bool idle,
                             float &activity) {
  if (input.size() != size_t(config.width)) throw std::invalid_argument("Invalid native input size");
  std::vector<float> packed(state_size());
  pack(state, packed.data());
  Vector hidden(config.width);
  advance_batch(input.data(), 1, packed.data(), idle, packed.data(), hidden.data(), &activity);
  state = unpack(packed.data());
  return hidden;
}

} // namespace neurogen::cortical
