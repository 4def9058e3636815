// Public C++ engine API of the B200 engine.  Same class and method names as
// the reference's include/engine/NeuralEngine.h:6-31; the C ABI it carries is
// declared in neurogen_b200.h.  Weights are uploaded to the current CUDA
// device once, at construction; every call runs there.
#pragma once
#include "CorticalColumnV2.h"
#include <cstdint>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

namespace ngb {
class DeviceModel; // GPU-resident weights, scratch and launch sequence
}
namespace neurogen::cortical {
struct EngineConfig {
  int columns, width, regions, ticks, idle_steps;
};
class NeuralEngine {
public:
  // backend must be "cuda"; anything else throws (no silent fallback).
  NeuralEngine(EngineConfig config, const float *weights, size_t count,
               const std::string &backend);
  ~NeuralEngine();
  size_t state_size() const;
  size_t parameter_count() const;
  // One region pass of every region (reference NeuralEngine::advance).
  Vector advance(const Vector &input, std::vector<ColumnState> &state, bool idle,
                 float &activity);
  // One token (reference NeuralEngine::step); returns the 264 logits.
  Vector step(int token, std::vector<ColumnState> &state, Vector &hidden,
              float &activity);
  std::vector<ColumnState> unpack(const float *state) const;
  void pack(const std::vector<ColumnState> &state, float *output) const;

  // Batched forms on packed host state [batch, state_size()].  state and
  // next_state may alias.  hidden/activity/logits may be null.
  void step_batch(const int *tokens, int batch, const float *state,
                  float *next_state, float *logits, float *hidden,
                  float *activity);
  void advance_batch(const float *inputs, int batch, const float *state,
                     bool idle, float *next_state, float *hidden,
                     float *activity);
  ngb::DeviceModel &device() { return *impl_; }

  EngineConfig config;
  std::string backend_name() const;
  std::mutex mutex;

private:
  std::unique_ptr<ngb::DeviceModel> impl_;
};
} // namespace neurogen::cortical
