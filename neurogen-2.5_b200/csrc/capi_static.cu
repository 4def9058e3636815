// ng_step_static: a token step whose device working memory is a fixed,
// file-scope array instead of buffers the library allocates.
//
// Who needs it: ng_step allocates its device working memory on first use and
// grows it when a larger batch arrives (cudaMalloc).  Some callers cannot
// allow that during a step: code running under a fixed device-memory budget
// set aside before streaming starts, and latency-critical streaming loops (a
// live token/audio stream) where a cudaMalloc may take the driver's
// allocation lock and implicitly synchronise the whole device.  This entry
// point never allocates: the state staging, the activations between kernels,
// the spike counters and the outputs all live in g_step_scratch below, a
// 1 MiB __device__ array that every GPU loading this library holds until the
// process exits.  The weights still live where ng_create put them; the
// caller still passes host inputs and outputs, exactly as for ng_step.
#include "capi_common.h"
#include "lang_engine.h"
#include "neurogen_b200.h"

#include <cuda_runtime.h>
#include <cmath>
#include <mutex>
#include <string>

using neurogen::cortical::NeuralEngine;

namespace ngb {
namespace {

// Capacity of the fixed working memory, in floats (1 MiB).  One BC-250 step
// (state 44,032 floats + activations) needs about 57k floats.
constexpr size_t kStepScratchFloats = size_t(1) << 18;

__device__ __align__(256) float g_step_scratch[kStepScratchFloats];

// Host copy of g_step_scratch's device address, looked up once per device.
// In host code the array's name is only a host-side stand-in, so kernels get
// this address, never `g_step_scratch` itself.
constexpr int kMaxDevices = 64;
float *g_scratch_addr[kMaxDevices] = {};
// Each device holds its own copy of the array, so calls are serialised per
// device: static steps on different GPUs run side by side.
std::mutex g_scratch_mutex[kMaxDevices];

// First call on a device (that device current): look the array up and load
// every language-core kernel, so that no later call makes the driver load
// code.  Must happen outside any stream capture.
float *scratch_address(int device) {
  if (device < 0 || device >= kMaxDevices) throw std::runtime_error("CUDA device index out of range");
  if (!g_scratch_addr[device]) {
    float *p = nullptr;
    cuda_check(cudaGetSymbolAddress(reinterpret_cast<void **>(&p), g_step_scratch),
               "cudaGetSymbolAddress(g_step_scratch)");
    preload_lang_kernels();
    g_scratch_addr[device] = p;
  }
  return g_scratch_addr[device];
}

// Offsets (in floats, 256-byte aligned) of one batch-1 step's buffers.
struct StepLayout {
  size_t state, token, h, hraw, vin, fb, tr, feat, cnt, logits, hidden, act, total;
  explicit StepLayout(const LangDims &d) {
    size_t at = 0;
    auto take = [&](size_t count) {
      const size_t off = at;
      at += (count + 63) & ~size_t(63);
      return off;
    };
    state = take(size_t(d.S));
    token = take(1);
    h = take(size_t(d.w));
    hraw = take(size_t(d.w));
    vin = take(size_t(d.c) * d.n_in);
    fb = take(size_t(d.R) * d.c * d.n_fb);
    tr = take(size_t(d.n));
    feat = take(size_t(d.c) * d.n_out * 2);
    cnt = take(size_t(1 + d.idle) * d.R);
    logits = take(kVocab);
    hidden = take(size_t(d.w));
    act = take(1);
    total = at;
  }
};

} // namespace
} // namespace ngb

using namespace ngb;

extern "C" int ng_step_static(void *p, int token, const float *state, size_t state_count, float *next_state,
                              float *logits, float *hidden, float *activity) {
  return guarded([&] {
    if (!p) throw std::invalid_argument("Null native engine");
    auto &e = *static_cast<NeuralEngine *>(p);
    if (!state || state_count != e.state_size()) throw std::invalid_argument("Invalid native state size");
    for (size_t i = 0; i < state_count; ++i)
      if (!std::isfinite(state[i])) throw std::invalid_argument("Non-finite native state");
    if (!next_state || !logits || !hidden || !activity) throw std::invalid_argument("Null output");
    if (token < 0 || token >= kVocab) throw std::invalid_argument("Token must be in 0..263");
    std::lock_guard<std::mutex> lock(e.mutex);
    DeviceModel &m = e.device();
    if (m.device < 0 || m.device >= kMaxDevices) throw std::runtime_error("CUDA device index out of range");
    std::lock_guard<std::mutex> scratch_lock(g_scratch_mutex[m.device]);
    const StepLayout L(m.dims);
    if (L.total > kStepScratchFloats)
      throw std::invalid_argument("ng_step_static: this model needs " + std::to_string(L.total) +
                                  " floats of device working memory, more than the fixed " +
                                  std::to_string(kStepScratchFloats) + "-float (1 MiB) buffer; use ng_step");
    NGB_CUDA(cudaSetDevice(m.device));
    float *base = scratch_address(m.device);
    ScratchView v{base + L.h, base + L.hraw, base + L.vin, base + L.fb, base + L.tr, base + L.feat,
                  reinterpret_cast<int *>(base + L.cnt)};
    float *d_state = base + L.state, *d_logits = base + L.logits, *d_hidden = base + L.hidden,
          *d_act = base + L.act;
    int *d_token = reinterpret_cast<int *>(base + L.token);
    const int w = m.dims.w, idle = m.dims.idle;
    cudaStream_t st = m.stream;
    NGB_CUDA(cudaMemcpyAsync(d_token, &token, sizeof(int), cudaMemcpyHostToDevice, st));
    NGB_CUDA(cudaMemcpyAsync(d_state, state, state_count * sizeof(float), cudaMemcpyHostToDevice, st));
    // enqueue_view zeroes the spike counters itself; nothing else is read
    // before it is written, so the previous call's contents do not matter.
    m.enqueue_view(1, d_token, nullptr, false, 1 + idle, d_state, d_logits, d_hidden, d_act, v, st);
    NGB_CUDA(cudaMemcpyAsync(next_state, d_state, state_count * sizeof(float), cudaMemcpyDeviceToHost, st));
    NGB_CUDA(cudaMemcpyAsync(logits, d_logits, kVocab * sizeof(float), cudaMemcpyDeviceToHost, st));
    NGB_CUDA(cudaMemcpyAsync(hidden, d_hidden, size_t(w) * sizeof(float), cudaMemcpyDeviceToHost, st));
    NGB_CUDA(cudaMemcpyAsync(activity, d_act, sizeof(float), cudaMemcpyDeviceToHost, st));
    NGB_CUDA(cudaStreamSynchronize(st));
    m.check_device_errors(); // same error reporting as ng_step
  });
}
