// C ABI of the language core (include/neurogen_b200.h, parts 1-3).  Same error
// convention as the reference's C ABI (src/native/NeuralEngine.cpp:193-267):
// exceptions become -1 / NULL plus a thread-local ng_error() message, and one
// mutex per engine serialises calls on a shared handle.
#include "capi_common.h"
#include "lang_engine.h"
#include "neurogen_b200.h"

#include <algorithm>
#include <cmath>
#include <mutex>

using neurogen::cortical::NeuralEngine;

namespace ngb {
thread_local std::string g_error;
thread_local std::string g_backend_label;

namespace {
NeuralEngine &checked(void *p, const float *state, size_t n) {
  if (!p) throw std::invalid_argument("Null native engine");
  auto &e = *static_cast<NeuralEngine *>(p);
  if (!state || n != e.state_size()) throw std::invalid_argument("Invalid native state size");
  return e;
}

// A device-resident pool of sessions sharing one engine's weights.
struct Pool {
  NeuralEngine *engine;
  int B;
  DeviceBuffer state, tokens, logits, hidden, act;
  Scratch sc;
  cudaStream_t stream = nullptr;
  cudaGraphExec_t graph = nullptr; // one token step of the whole pool
  std::mutex mu;
  ~Pool() {
    if (graph) cudaGraphExecDestroy(graph);
    if (stream) cudaStreamDestroy(stream);
  }
  // Enqueue one token step reading `tokens` and writing logits/hidden/act
  // into the pool's own buffers.  The step is captured into a CUDA graph on
  // first use and replayed afterwards (its buffers never move).
  void token_step(cudaStream_t st) {
    if (!graph) {
      const DeviceModel &m = engine->device();
      cudaGraph_t g = nullptr;
      NGB_CUDA(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
      try {
        m.enqueue(B, tokens.as<int>(), nullptr, false, 1 + engine->config.idle_steps, state.as<float>(),
                  logits.as<float>(), hidden.as<float>(), act.as<float>(), sc, stream);
      } catch (...) {
        cudaStreamEndCapture(stream, &g);
        if (g) cudaGraphDestroy(g);
        throw;
      }
      NGB_CUDA(cudaStreamEndCapture(stream, &g));
      const cudaError_t e = cudaGraphInstantiate(&graph, g, 0);
      cudaGraphDestroy(g);
      cuda_check(e, "cudaGraphInstantiate");
    }
    NGB_CUDA(cudaGraphLaunch(graph, st));
  }
};
} // namespace
} // namespace ngb

using namespace ngb;

extern "C" {

void *ng_create(int c, int w, int r, int t, int idle, const float *weights, size_t n, const char *backend) {
  return guarded_ptr([&]() -> void * {
    return new NeuralEngine({c, w, r, t, idle}, weights, n, backend ? backend : "cuda");
  });
}

void ng_destroy(void *e) { delete static_cast<NeuralEngine *>(e); }

const char *ng_error(void) { return g_error.c_str(); }

const char *ng_backend(void *e) {
  if (!e) return "invalid";
  g_backend_label = static_cast<NeuralEngine *>(e)->backend_name();
  return g_backend_label.c_str();
}

int ng_step(void *p, int token, const float *s, size_t n, float *next, float *logits, float *h, float *a) {
  return guarded([&] {
    auto &e = checked(p, s, n);
    std::lock_guard<std::mutex> lock(e.mutex);
    if (!next || !logits || !h || !a) throw std::invalid_argument("Null output");
    e.step_batch(&token, 1, s, next, logits, h, a);
  });
}

int ng_advance(void *p, const float *input, const float *s, size_t n, int idle, float *next, float *h,
               float *a) {
  return guarded([&] {
    auto &e = checked(p, s, n);
    std::lock_guard<std::mutex> lock(e.mutex);
    if (!input || !next || !h || !a) throw std::invalid_argument("Null input/output");
    e.advance_batch(input, 1, s, idle != 0, next, h, a);
  });
}

size_t ng_state_size(void *p) { return p ? static_cast<NeuralEngine *>(p)->state_size() : 0; }

size_t ng_parameter_count(int columns, int width, int regions) {
  neurogen::cortical::CorticalColumnV2 col({columns, width, 1});
  return 528ull * width + kVocab + size_t(regions) * col.parameter_count();
}

int ng_step_batch(void *p, const int *tokens, int batch, const float *s, size_t n, float *next,
                  float *logits, float *h, float *a) {
  return guarded([&] {
    auto &e = checked(p, s, n);
    std::lock_guard<std::mutex> lock(e.mutex);
    if (!next || !logits || !h || !a) throw std::invalid_argument("Null output");
    e.step_batch(tokens, batch, s, next, logits, h, a);
  });
}

int ng_advance_batch(void *p, const float *inputs, int batch, const float *s, size_t n, int idle,
                     float *next, float *h, float *a) {
  return guarded([&] {
    auto &e = checked(p, s, n);
    std::lock_guard<std::mutex> lock(e.mutex);
    if (!next || !h || !a) throw std::invalid_argument("Null output");
    e.advance_batch(inputs, batch, s, idle != 0, next, h, a);
  });
}

void *ng_pool_create(void *engine, int batch) {
  return guarded_ptr([&]() -> void * {
    if (!engine) throw std::invalid_argument("Null native engine");
    if (batch < 1) throw std::invalid_argument("Need at least one batch item");
    auto *e = static_cast<NeuralEngine *>(engine);
    DeviceModel &m = e->device();
    NGB_CUDA(cudaSetDevice(m.device));
    auto pool = std::make_unique<Pool>();
    pool->engine = e;
    pool->B = batch;
    const size_t S = e->state_size();
    pool->state.reset(S * batch * 4);
    NGB_CUDA(cudaMemset(pool->state.as<float>(), 0, S * batch * 4));
    pool->tokens.reset(batch * sizeof(int));
    pool->logits.reset(size_t(batch) * kVocab * 4);
    pool->hidden.reset(size_t(batch) * e->config.width * 4);
    pool->act.reset(size_t(batch) * 4);
    pool->sc.ensure(m.dims, batch, m.tc_proj);
    NGB_CUDA(cudaStreamCreateWithFlags(&pool->stream, cudaStreamNonBlocking));
    return pool.release();
  });
}

void ng_pool_destroy(void *p) { delete static_cast<Pool *>(p); }

int ng_pool_load(void *p, const float *state) {
  return guarded([&] {
    if (!p || !state) throw std::invalid_argument("Null pool or state");
    auto &pool = *static_cast<Pool *>(p);
    std::lock_guard<std::mutex> lock(pool.mu);
    const size_t count = pool.engine->state_size() * pool.B;
    for (size_t i = 0; i < count; ++i)
      if (!std::isfinite(state[i])) throw std::invalid_argument("Non-finite native state");
    NGB_CUDA(cudaSetDevice(pool.engine->device().device));
    NGB_CUDA(cudaMemcpy(pool.state.as<float>(), state, count * 4, cudaMemcpyHostToDevice));
  });
}

int ng_pool_store(void *p, float *state) {
  return guarded([&] {
    if (!p || !state) throw std::invalid_argument("Null pool or state");
    auto &pool = *static_cast<Pool *>(p);
    std::lock_guard<std::mutex> lock(pool.mu);
    NGB_CUDA(cudaSetDevice(pool.engine->device().device));
    NGB_CUDA(cudaStreamSynchronize(pool.stream));
    NGB_CUDA(cudaMemcpy(state, pool.state.as<float>(), pool.engine->state_size() * pool.B * 4,
                        cudaMemcpyDeviceToHost));
  });
}

int ng_pool_step(void *p, const int *tokens, float *logits, float *hidden, float *activity) {
  return guarded([&] {
    if (!p || !tokens) throw std::invalid_argument("Null pool or tokens");
    auto &pool = *static_cast<Pool *>(p);
    std::lock_guard<std::mutex> lock(pool.mu);
    for (int b = 0; b < pool.B; ++b)
      if (tokens[b] < 0 || tokens[b] >= kVocab) throw std::invalid_argument("Token must be in 0..263");
    DeviceModel &m = pool.engine->device();
    NGB_CUDA(cudaSetDevice(m.device));
    cudaStream_t st = pool.stream;
    const int B = pool.B, w = pool.engine->config.width;
    NGB_CUDA(cudaMemcpyAsync(pool.tokens.as<int>(), tokens, B * sizeof(int), cudaMemcpyHostToDevice, st));
    pool.token_step(st);
    if (logits)
      NGB_CUDA(cudaMemcpyAsync(logits, pool.logits.as<float>(), size_t(B) * kVocab * 4, cudaMemcpyDeviceToHost, st));
    if (hidden)
      NGB_CUDA(cudaMemcpyAsync(hidden, pool.hidden.as<float>(), size_t(B) * w * 4, cudaMemcpyDeviceToHost, st));
    if (activity)
      NGB_CUDA(cudaMemcpyAsync(activity, pool.act.as<float>(), size_t(B) * 4, cudaMemcpyDeviceToHost, st));
    NGB_CUDA(cudaStreamSynchronize(st));
    m.check_device_errors();
  });
}

int ng_pool_step_device(void *p, const int *d_tokens, float *d_logits, void *stream) {
  return guarded([&] {
    if (!p || !d_tokens) throw std::invalid_argument("Null pool or tokens");
    auto &pool = *static_cast<Pool *>(p);
    std::lock_guard<std::mutex> lock(pool.mu);
    DeviceModel &m = pool.engine->device();
    NGB_CUDA(cudaSetDevice(m.device));
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : pool.stream;
    NGB_CUDA(cudaMemcpyAsync(pool.tokens.as<int>(), d_tokens, pool.B * sizeof(int), cudaMemcpyDeviceToDevice, st));
    pool.token_step(st);
    if (d_logits)
      NGB_CUDA(cudaMemcpyAsync(d_logits, pool.logits.as<float>(), size_t(pool.B) * kVocab * 4,
                               cudaMemcpyDeviceToDevice, st));
  });
}

float *ng_pool_device_state(void *p) { return p ? static_cast<Pool *>(p)->state.as<float>() : nullptr; }

} // extern "C"
