// Public C++ column types of the B200 engine (reference interface:
// include/engine/CorticalColumnV2.h:9-44).  A column region here is a
// description of one region's sizes and unit tables; its weights live on the
// GPU inside NeuralEngine, so there is no per-call ComputeBackend.
#pragma once
#include "ALIFNeuron.h"
#include <cstddef>
#include <string>
#include <vector>

namespace neurogen::cortical {
using Vector = std::vector<float>;
struct CorticalColumnConfig {
  int columns = 1, width = 32, ticks = 2;
};
// Caller-owned state of one region (host side).
struct ColumnState {
  ALIFNeuronArrays neurons;
  Vector memory;
  ColumnState(size_t n, size_t w) : neurons(n), memory(w) {}
};
class CorticalColumnV2 {
public:
  explicit CorticalColumnV2(CorticalColumnConfig config);
  // Number of packed fp32 parameters of one region (reference
  // CorticalColumnV2::parameter_count, src/native/NeuralEngine.cpp:32-37).
  size_t parameter_count() const;
  const CorticalColumnConfig &config() const { return config_; }
  // Unit tables of a 64-unit column: sign (+1 E / -1 I), layer, and the ids
  // that receive input, receive feedback, and are read out.
  const std::vector<float> &sign() const { return sign_; }
  const std::vector<int> &layer() const { return layer_; }
  const std::vector<int> &input_ids() const { return input_ids_; }
  const std::vector<int> &feedback_ids() const { return feedback_ids_; }
  const std::vector<int> &output_ids() const { return output_ids_; }

private:
  CorticalColumnConfig config_;
  std::vector<float> sign_;
  std::vector<int> layer_, input_ids_, feedback_ids_, output_ids_;
};
} // namespace neurogen::cortical
