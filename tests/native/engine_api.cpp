// C++ caller of the public engine API (include/engine/*.h), written the way a
// program against the reference's headers is (reference tests/native/smoke.cpp:
// build engines, step tokens, compare states and logits).  The comparison side
// is the reference's own native CPU library, loaded at run time through its C
// ABI (argv[1]: path of that library); this library has no CPU backend.
//
//   engine_api <reference library> [check|compile-only]
//
// Checks, for the configuration {columns 3, width 17, regions 2, ticks 3,
// idle 1} with seeded non-uniform weights:
//   1. NeuralEngine(..., "cuda"): 12 token steps through the C++ step/pack/unpack
//      API, state and logits within 1e-4 of the reference (the bar of the
//      reference's own smoke test), spikes identical;
//   2. CorticalColumnV2::load / step through make_backend("cuda"): each region
//      loaded from the packed stream and stepped as the reference engine's
//      advance does; 12 token steps bit-identical to the reference library;
//   3. make_backend("cpu") and NeuralEngine(..., "cpu") are refused.
#include "engine/NeuralEngine.h"

#include <dlfcn.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <iostream>
#include <stdexcept>
#include <string>
#include <vector>

using namespace neurogen::cortical;

namespace {
using CreateFn = void *(*)(int, int, int, int, int, const float *, size_t, const char *);
using StepFn = int (*)(void *, int, const float *, size_t, float *, float *, float *, float *);
using ErrorFn = const char *(*)();

struct Reference {
  void *lib = nullptr, *engine = nullptr;
  StepFn step = nullptr;
  Reference(const char *path, EngineConfig c, const std::vector<float> &w) {
    // DEEPBIND: the reference library's C++ classes have the same names as this
    // library's (the same public API), so it must bind to its own definitions.
    lib = dlopen(path, RTLD_NOW | RTLD_LOCAL | RTLD_DEEPBIND);
    if (!lib) throw std::runtime_error(std::string("cannot load the reference library: ") + dlerror());
    auto create = reinterpret_cast<CreateFn>(dlsym(lib, "ng_create"));
    step = reinterpret_cast<StepFn>(dlsym(lib, "ng_step"));
    auto error = reinterpret_cast<ErrorFn>(dlsym(lib, "ng_error"));
    if (!create || !step || !error) throw std::runtime_error("reference library lacks the C ABI");
    engine = create(c.columns, c.width, c.regions, c.ticks, c.idle_steps, w.data(), w.size(), "cpu");
    if (!engine) throw std::runtime_error(std::string("reference ng_create: ") + error());
  }
};

std::vector<float> weights_for(const EngineConfig &c, size_t count) {
  // Deterministic non-uniform weights (a 32-bit LCG), so recurrent ticks spike.
  std::vector<float> w(count);
  uint32_t s = 12345u;
  for (float &x : w) {
    s = s * 1664525u + 1013904223u;
    x = (float(s >> 8) / float(1u << 24) - .5f) * .6f;
  }
  (void)c;
  return w;
}

void check_close(const std::vector<float> &a, const std::vector<float> &b, float tol, const char *what) {
  for (size_t j = 0; j < a.size(); ++j)
    if (!std::isfinite(a[j]) || std::abs(a[j] - b[j]) > tol)
      throw std::runtime_error(std::string(what) + " mismatch at " + std::to_string(j));
}
}  // namespace

int main(int argc, char **argv) {
  if (argc < 2) {
    std::cerr << "usage: engine_api <reference library> [check]\n";
    return 2;
  }
  try {
    const EngineConfig c{3, 17, 2, 3, 1};
    CorticalColumnV2 probe({c.columns, c.width, c.ticks});
    const size_t count = 528 * size_t(c.width) + 264 + size_t(c.regions) * probe.parameter_count();
    const std::vector<float> w = weights_for(c, count);
    Reference ref(argv[1], c, w);

    // 1. The engine API on the GPU.
    NeuralEngine cuda(c, w.data(), w.size(), "cuda");
    if (cuda.backend_name().rfind("cuda", 0) != 0) throw std::runtime_error("unexpected backend " + cuda.backend_name());
    if (cuda.parameter_count() != count) throw std::runtime_error("parameter count");
    const size_t S = cuda.state_size();
    std::vector<float> zero(S), rs(S), rnext(S), rl(264), rh(c.width), ra(1);
    auto state = cuda.unpack(zero.data());
    rs = zero;
    for (int i = 0; i < 12; ++i) {
      const int token = i == 0 ? 257 : 40 + 7 * i;
      Vector hidden;
      float act = 0;
      const Vector logits = cuda.step(token, state, hidden, act);
      if (ref.step(ref.engine, token, rs.data(), S, rnext.data(), rl.data(), rh.data(), ra.data()))
        throw std::runtime_error("reference step failed");
      rs = rnext;
      std::vector<float> packed(S);
      cuda.pack(state, packed.data());
      check_close(packed, rs, 1e-4f, "engine state");
      check_close(logits, rl, 1e-4f, "engine logits");
      for (size_t r = 0; r < size_t(c.regions); ++r)
        if (state[r].neurons.last_spikes != std::vector<float>(rs.begin() + r * (S / c.regions) + 3 * c.columns * 64,
                                                               rs.begin() + r * (S / c.regions) + 4 * c.columns * 64))
          throw std::runtime_error("engine spikes differ");
    }

    // 2. The column API through a CUDA ComputeBackend, stepped as the engine's advance.
    auto backend = make_backend("cuda");
    const float *p = w.data();
    const Vector embedding(p, p + 264 * size_t(c.width));
    p += 264 * size_t(c.width);
    std::vector<CorticalColumnV2> regions;
    for (int r = 0; r < c.regions; ++r) {
      regions.emplace_back(CorticalColumnConfig{c.columns, c.width, c.ticks});
      regions.back().load(p);
    }
    const Vector head(p, p + 264 * size_t(c.width));
    p += 264 * size_t(c.width);
    const Vector head_bias(p, p + 264);
    p += 264;
    if (p != w.data() + w.size()) throw std::runtime_error("column loads did not consume the stream");
    auto cstate = cuda.unpack(zero.data());
    rs = zero;
    auto advance = [&](const Vector &input, bool idle, float &activity) {
      Vector h = input;
      activity = 0;
      for (int r = 0; r < c.regions; ++r) {
        float a = 0;
        h = regions[r].step(h, cstate[r], !idle || r > 0, *backend, a);
        activity += a;
      }
      activity /= c.regions;
      return h;
    };
    for (int i = 0; i < 12; ++i) {
      const int token = i == 0 ? 257 : 40 + 7 * i;
      float act = 0;
      Vector h = advance(Vector(embedding.begin() + token * c.width, embedding.begin() + (token + 1) * c.width),
                         false, act);
      for (int k = 0; k < c.idle_steps; ++k) {
        float a = 0;
        h = advance(Vector(c.width), true, a);
        act += a;
      }
      const Vector logits = backend->matvec(head, h, head_bias);
      if (ref.step(ref.engine, token, rs.data(), S, rnext.data(), rl.data(), rh.data(), ra.data()))
        throw std::runtime_error("reference step failed");
      rs = rnext;
      std::vector<float> packed(S);
      cuda.pack(cstate, packed.data());
      if (std::memcmp(packed.data(), rs.data(), S * 4) != 0) throw std::runtime_error("column state not bit-identical");
      if (std::memcmp(logits.data(), rl.data(), 264 * 4) != 0) throw std::runtime_error("column logits not bit-identical");
      if (act / (1 + c.idle_steps) != ra[0]) throw std::runtime_error("column activity differs");
    }

    // 3. No CPU backend.
    bool refused = false;
    try {
      make_backend("cpu");
    } catch (const std::invalid_argument &e) {
      refused = std::string(e.what()).find("unavailable") != std::string::npos;
    }
    if (!refused) throw std::runtime_error("make_backend(\"cpu\") was not refused");
    refused = false;
    try {
      NeuralEngine cpu(c, w.data(), w.size(), "cpu");
    } catch (const std::invalid_argument &e) {
      refused = std::string(e.what()).find("no silent fallback") != std::string::npos;
    }
    if (!refused) throw std::runtime_error("a \"cpu\" engine was not refused");
    std::cout << "Passed: " << cuda.backend_name() << " (engine API within 1e-4, column API bit-identical)\n";
  } catch (const std::exception &e) {
    std::cerr << e.what() << "\n";
    return 1;
  }
  return 0;
}
