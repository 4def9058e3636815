// Public C++ column types of the B200 engine (reference interface:
// include/engine/CorticalColumnV2.h:9-44).  NeuralEngine (NeuralEngine.h) is
// the fast path: all regions' weights resident on the GPU, one launch
// sequence per token.  The column-level API below keeps the reference's
// per-call boundary for C++ callers written against it: a CorticalColumnV2
// loads one region from the packed stream and steps it through a
// ComputeBackend, whose projections and recurrent ticks run on the GPU.
#pragma once
#include "ALIFNeuron.h"
#include <cstddef>
#include <memory>
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

// The per-call compute boundary of one region (reference
// CorticalColumnV2.h:20-28): a dense projection y = W x + b (W row-major,
// rows = W.size() / x.size(), b empty = zero) and `ticks` synchronous
// recurrent ALIF ticks of the region's units driven by `current`, returning
// the spikes per unit per tick.  Both are exact in the reference's fp32
// operation order.
class ComputeBackend {
public:
  virtual ~ComputeBackend() = default;
  virtual Vector matvec(const Vector &weights, const Vector &x, const Vector &bias) = 0;
  virtual float ticks(ALIFNeuronArrays &, const Vector &current, const Vector &weights, const Vector &sign,
                      int ticks) = 0;
  virtual std::string name() const = 0;
};
// "cuda" -> a backend on the current CUDA device (an sm_100 GPU is required).
// Any other name throws std::invalid_argument (no silent fallback).
std::unique_ptr<ComputeBackend> make_backend(const std::string &name);

class CorticalColumnV2 {
public:
  explicit CorticalColumnV2(CorticalColumnConfig config);
  // Reads this region's parameters from the packed stream and advances
  // `data` past them (reference CorticalColumnV2::load).
  void load(const float *&data);
  // One region step (reference CorticalColumnV2::step): input and feedback
  // currents, the recurrent ticks on `backend`, the readout, LayerNorm and the
  // memory update.  Returns the region's output h; updates `state`.
  Vector step(const Vector &input, ColumnState &state, bool sensory, ComputeBackend &backend,
              float &activity) const;
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
  // Gain of each recurrent connection of a column [post][pre]: the presynaptic
  // sign where the laminar connectivity rule allows the pair, else 0.
  std::vector<float> recurrent_gain() const;

private:
  CorticalColumnConfig config_;
  std::vector<float> sign_;
  std::vector<int> layer_, input_ids_, feedback_ids_, output_ids_;
  // Loaded parameters (host copies; transformed as the model defines them).
  Vector weights_, input_, input_bias_, feedback_, output_, output_bias_, norm_, norm_bias_, decay_;
};
} // namespace neurogen::cortical
