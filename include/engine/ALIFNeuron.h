// Public C++ neuron types of the B200 engine.  Same names and fields as the
// reference's include/engine/ALIFNeuron.h:8-17 so C++ callers compile unchanged.
#pragma once
#include <cstddef>
#include <vector>

namespace neurogen::cortical {
// Host-side structure-of-arrays view of one region's spiking units: the five
// per-unit state fields of the normalised ALIF language model.
struct ALIFNeuronArrays {
  std::vector<float> voltage, trace, adaptation, last_spikes, counts;
  explicit ALIFNeuronArrays(size_t n = 0)
      : voltage(n), trace(n), adaptation(n), last_spikes(n), counts(n) {}
};
// One laminar layer of a 64-unit column: layer number, E count, I count.
struct LayerParams {
  int layer, excitatory, inhibitory;
};
// The column's laminar table (64 units, 50 excitatory).
inline constexpr LayerParams layers[] = {{1, 0, 2},  {2, 8, 2},  {3, 8, 2},
                                         {4, 12, 3}, {5, 12, 3}, {6, 10, 2}};
} // namespace neurogen::cortical
