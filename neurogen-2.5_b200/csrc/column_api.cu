// Column-level C++ API: CorticalColumnV2::load / step through a ComputeBackend
// (reference include/engine/CorticalColumnV2.h:20-44, implementation
// src/native/NeuralEngine.cpp:38-110, backend contract
// src/native/PackedBackend.h:16-54 and src/native/CPUBackend.cpp:9-67).
//
// This is the per-call boundary of the reference, kept for C++ callers that
// drive one region at a time.  Each backend call copies its operands to the
// GPU, runs one kernel and copies the result back, as the reference's CUDA
// backend does; the fast path for whole tokens is NeuralEngine (weights
// resident on the device, one launch sequence per token).
//
// Numerics: the projection is one sequential fp32 chain per row starting from
// the bias, the tick is the reference's per-unit update, every operation
// rounded as written (this file is compiled with -fmad=false), and the
// sigmoid/tanh/LayerNorm of the column step run on the host with the same
// libm the reference calls -- so a region step is bit-identical to the
// reference's CPU backend.
#include "engine/CorticalColumnV2.h"
#include "common.h"

#include <algorithm>
#include <cmath>
#include <stdexcept>

namespace ngb {
namespace {

// y[i] = b[i] + sum_j W[i][j] x[j], j in order.  x staged in shared memory in
// pieces; one thread per row.
constexpr int MV_T = 128, MV_X = 2048;
__global__ void __launch_bounds__(MV_T) k_api_matvec(const float *W, const float *x, const float *b, float *y,
                                                     int rows, int cols) {
  __shared__ float xs[MV_X];
  const int i = blockIdx.x * MV_T + threadIdx.x;
  float v = (i < rows && b) ? b[i] : 0.f;
  for (int j0 = 0; j0 < cols; j0 += MV_X) {
    const int jn = min(MV_X, cols - j0);
    __syncthreads();
    for (int j = threadIdx.x; j < jn; j += MV_T) xs[j] = x[j0 + j];
    __syncthreads();
    if (i < rows) {
      const float *w = W + (size_t)i * cols + j0;
      for (int j = 0; j < jn; ++j) v = __fadd_rn(v, __fmul_rn(w[j], xs[j]));
    }
  }
  if (i < rows) y[i] = v;
}

// One synchronous tick of n units (n/64 columns): reads state `x`
// [V, trace, adaptation, last, counts] (5n), writes `y` (5n); spike total into
// *spikes.  Unit i = col*64 + id; recurrent input from the column's traces in
// presynaptic order; excitatory units add the traces of the same unit id in
// the neighbouring columns.
__global__ void __launch_bounds__(64) k_api_tick(const float *x, float *y, const float *current, const float *w,
                                                 const float *sign, int n, unsigned long long *spikes) {
  const int col = blockIdx.x, id = threadIdx.x, i = col * 64 + id;
  const bool exc = sign[id] > 0.f;
  const float *trace = x + n;
  float recurrent = 0.f;
  for (int j = 0; j < 64; ++j)
    recurrent = __fadd_rn(recurrent, __fmul_rn(w[(size_t)col * 4096 + id * 64 + j], trace[col * 64 + j]));
  float neighbor = 0.f;
  if (exc) {
    if (col > 0) neighbor = neighbor + trace[i - 64];
    if (i + 64 < n) neighbor = neighbor + trace[i + 64];
  }
  const float decay = exc ? .6f : .4f;
  const float voltage = decay * x[i] + (1 - decay) * (current[i] + recurrent + .08f * neighbor);
  const float spike = (voltage - (exc ? 1.f : .6f) - x[2 * n + i] >= 0 ? 1.f : 0.f) * (1 - x[3 * n + i]);
  y[i] = voltage * (1 - spike);
  y[n + i] = .8f * x[n + i] + .2f * spike;
  y[2 * n + i] = .98f * x[2 * n + i] + (exc ? .03f : 0.f) * spike;
  y[3 * n + i] = spike;
  y[4 * n + i] = x[4 * n + i] + spike;
  const unsigned fired = __ballot_sync(0xffffffffu, spike != 0.f);
  if ((id & 31) == 0 && fired) atomicAdd(spikes, (unsigned long long)__popc(fired));
}

// Grow-only device buffer.
struct Grow {
  DeviceBuffer buf;
  template <class T> T *at_least(size_t count) {
    if (buf.bytes() < count * sizeof(T)) buf.reset(count * sizeof(T));
    return buf.as<T>();
  }
};

class CudaBackend final : public neurogen::cortical::ComputeBackend {
public:
  CudaBackend() {
    device_ = require_sm100_device();
    label_ = device_label(device_);
    NGB_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
  }
  ~CudaBackend() override {
    if (stream_) cudaStreamDestroy(stream_);
  }
  std::string name() const override { return label_; }

  neurogen::cortical::Vector matvec(const neurogen::cortical::Vector &weights, const neurogen::cortical::Vector &x,
                                    const neurogen::cortical::Vector &bias) override {
    if (x.empty() || weights.size() % x.size()) throw std::invalid_argument("matvec: weights are not rows of x");
    const size_t rows = weights.size() / x.size();
    if (!bias.empty() && bias.size() != rows) throw std::invalid_argument("matvec: bias size differs from rows");
    NGB_CUDA(cudaSetDevice(device_));
    float *dw = w_.at_least<float>(weights.size()), *dx = x_.at_least<float>(x.size());
    float *db = bias.empty() ? nullptr : b_.at_least<float>(rows), *dy = y_.at_least<float>(rows);
    NGB_CUDA(cudaMemcpyAsync(dw, weights.data(), weights.size() * 4, cudaMemcpyHostToDevice, stream_));
    NGB_CUDA(cudaMemcpyAsync(dx, x.data(), x.size() * 4, cudaMemcpyHostToDevice, stream_));
    if (db) NGB_CUDA(cudaMemcpyAsync(db, bias.data(), rows * 4, cudaMemcpyHostToDevice, stream_));
    k_api_matvec<<<unsigned((rows + MV_T - 1) / MV_T), MV_T, 0, stream_>>>(dw, dx, db, dy, int(rows), int(x.size()));
    NGB_CUDA(cudaGetLastError());
    neurogen::cortical::Vector y(rows);
    NGB_CUDA(cudaMemcpyAsync(y.data(), dy, rows * 4, cudaMemcpyDeviceToHost, stream_));
    NGB_CUDA(cudaStreamSynchronize(stream_));
    return y;
  }

  float ticks(neurogen::cortical::ALIFNeuronArrays &s, const neurogen::cortical::Vector &current,
              const neurogen::cortical::Vector &weights, const neurogen::cortical::Vector &sign, int count) override {
    const size_t n = s.voltage.size();
    if (n == 0 || n % 64 || current.size() != n || weights.size() != n * 64 || sign.size() != 64 ||
        s.trace.size() != n || s.adaptation.size() != n || s.last_spikes.size() != n || s.counts.size() != n)
      throw std::invalid_argument("ticks: inconsistent neuron array sizes");
    if (count < 1) throw std::invalid_argument("ticks: count must be positive");
    NGB_CUDA(cudaSetDevice(device_));
    float *st = state_.at_least<float>(10 * n), *cur = cur_.at_least<float>(n), *dw = w_.at_least<float>(n * 64);
    float *sg = sign_.at_least<float>(64);
    unsigned long long *spk = spikes_.at_least<unsigned long long>(1);
    std::vector<float *> fields = {s.voltage.data(), s.trace.data(), s.adaptation.data(), s.last_spikes.data(),
                                   s.counts.data()};
    for (size_t f = 0; f < 5; ++f)
      NGB_CUDA(cudaMemcpyAsync(st + f * n, fields[f], n * 4, cudaMemcpyHostToDevice, stream_));
    NGB_CUDA(cudaMemcpyAsync(cur, current.data(), n * 4, cudaMemcpyHostToDevice, stream_));
    NGB_CUDA(cudaMemcpyAsync(dw, weights.data(), n * 64 * 4, cudaMemcpyHostToDevice, stream_));
    NGB_CUDA(cudaMemcpyAsync(sg, sign.data(), 64 * 4, cudaMemcpyHostToDevice, stream_));
    NGB_CUDA(cudaMemsetAsync(spk, 0, 8, stream_));
    for (int t = 0; t < count; ++t) {
      const float *in = st + size_t(t & 1) * 5 * n;
      float *out = st + size_t((t + 1) & 1) * 5 * n;
      k_api_tick<<<unsigned(n / 64), 64, 0, stream_>>>(in, out, cur, dw, sg, int(n), spk);
      NGB_CUDA(cudaGetLastError());
    }
    const float *fin = st + size_t(count & 1) * 5 * n;
    for (size_t f = 0; f < 5; ++f)
      NGB_CUDA(cudaMemcpyAsync(fields[f], fin + f * n, n * 4, cudaMemcpyDeviceToHost, stream_));
    unsigned long long total = 0;
    NGB_CUDA(cudaMemcpyAsync(&total, spk, 8, cudaMemcpyDeviceToHost, stream_));
    NGB_CUDA(cudaStreamSynchronize(stream_));
    // The reference sums the 0/1 spikes into a double: an exact integer count.
    return static_cast<float>(double(total) / (double(n) * count));
  }

private:
  int device_ = 0;
  std::string label_;
  cudaStream_t stream_ = nullptr;
  Grow w_, x_, b_, y_, state_, cur_, sign_, spikes_;
};

float sigmoid_host(float x) { return 1.f / (1.f + std::exp(-x)); }

neurogen::cortical::Vector take(const float *&data, size_t count) {
  neurogen::cortical::Vector v(data, data + count);
  data += count;
  return v;
}

} // namespace
} // namespace ngb

namespace neurogen::cortical {

std::unique_ptr<ComputeBackend> make_backend(const std::string &name) {
  if (name == "cuda") return std::make_unique<ngb::CudaBackend>();
  throw std::invalid_argument("Native backend '" + name +
                              "' unavailable; this library provides only 'cuda' (B200, sm_100a) (no silent fallback)");
}

// Laminar connectivity: same layer, one of the preferred feed-forward pairs
// (4->2, 4->3, 2->3, 3->5, 5->6, 6->4), or an inhibitory presynaptic cell
// within one layer; no autapses (src/native/NeuralEngine.cpp:41-56).
std::vector<float> CorticalColumnV2::recurrent_gain() const {
  static const int preferred[6][2] = {{4, 2}, {4, 3}, {2, 3}, {3, 5}, {5, 6}, {6, 4}};
  std::vector<float> gain(64 * 64, 0.f);
  for (int post = 0; post < 64; ++post)
    for (int pre = 0; pre < 64; ++pre) {
      const int lp = layer_[pre], lq = layer_[post];
      bool ok = lp == lq;
      for (const auto &pr : preferred) ok = ok || (lp == pr[0] && lq == pr[1]);
      ok = ok || (sign_[pre] < 0 && std::abs(lq - lp) <= 1);
      gain[post * 64 + pre] = (ok && post != pre) ? sign_[pre] : 0.f;
    }
  return gain;
}

void CorticalColumnV2::load(const float *&data) {
  if (!data) throw std::invalid_argument("Null weights");
  const size_t c = config_.columns, w = config_.width;
  const std::vector<float> gain = recurrent_gain();
  weights_ = ngb::take(data, c * 4096);
  // softplus(raw) * gain, with the host libm as the reference loader.
  for (size_t col = 0; col < c; ++col)
    for (int k = 0; k < 4096; ++k) {
      float &x = weights_[col * 4096 + k];
      x = gain[k] != 0.f ? (std::max(x, 0.f) + std::log1p(std::exp(-std::abs(x)))) * gain[k] : 0.f;
    }
  input_ = ngb::take(data, c * input_ids_.size() * w);
  input_bias_ = ngb::take(data, c * input_ids_.size());
  feedback_ = ngb::take(data, c * feedback_ids_.size() * w);
  output_ = ngb::take(data, w * c * output_ids_.size() * 2);
  output_bias_ = ngb::take(data, w);
  norm_ = ngb::take(data, w);
  norm_bias_ = ngb::take(data, w);
  decay_ = ngb::take(data, w);
  for (float &d : decay_) d = .5f + .499f * ngb::sigmoid_host(d);
}

Vector CorticalColumnV2::step(const Vector &input, ColumnState &state, bool sensory, ComputeBackend &backend,
                              float &activity) const {
  const size_t c = config_.columns, w = config_.width, n = c * 64;
  const size_t n_in = input_ids_.size(), n_fb = feedback_ids_.size();
  if (weights_.size() != c * 4096) throw std::logic_error("CorticalColumnV2::step before load");
  if (state.neurons.voltage.size() != n || state.memory.size() != w)
    throw std::invalid_argument("Invalid native region state");
  if (sensory && input.size() != w) throw std::invalid_argument("Invalid native input size");
  // Baseline drive, then the sensory input of the layer-4 excitatory cells
  // and the feedback of layers 1, 5 and 6.
  Vector current(n);
  for (size_t i = 0; i < n; ++i) current[i] = sign_[i % 64] > 0 ? .15f : .35f;
  if (sensory) {
    const Vector v = backend.matvec(input_, input, input_bias_);
    for (size_t col = 0; col < c; ++col)
      for (size_t j = 0; j < n_in; ++j)
        current[col * 64 + input_ids_[j]] = 3 * ngb::sigmoid_host(v[col * n_in + j]);
  }
  const Vector fb = backend.matvec(feedback_, state.memory, {});
  for (size_t col = 0; col < c; ++col)
    for (size_t j = 0; j < n_fb; ++j)
      current[col * 64 + feedback_ids_[j]] += .5f * std::tanh(fb[col * n_fb + j]);
  activity = backend.ticks(state.neurons, current, weights_, sign_, config_.ticks);
  // Readout features: voltages then traces of the excitatory cells, column by column.
  Vector features;
  features.reserve(2 * c * output_ids_.size());
  for (const Vector *field : {&state.neurons.voltage, &state.neurons.trace})
    for (size_t col = 0; col < c; ++col)
      for (int id : output_ids_) features.push_back((*field)[col * 64 + id]);
  Vector h = backend.matvec(output_, features, output_bias_);
  // LayerNorm of h + 0.25 * memory (statistics in double), then the memory update.
  double mean = 0, var = 0;
  for (size_t i = 0; i < w; ++i) {
    h[i] += .25f * state.memory[i];
    mean += h[i];
  }
  mean /= double(w);
  for (float v : h) var += (v - mean) * (v - mean);
  const float inv = 1.f / std::sqrt(var / double(w) + 1e-5);
  for (size_t i = 0; i < w; ++i) {
    h[i] = (h[i] - static_cast<float>(mean)) * inv * norm_[i] + norm_bias_[i];
    state.memory[i] = decay_[i] * state.memory[i] + (1 - decay_[i]) * h[i];
  }
  return h;
}

} // namespace neurogen::cortical
