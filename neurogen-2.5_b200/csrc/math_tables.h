// Host-built exception tables that make the device's tanh and sigmoid return
// the host C library's values (libm_match.cuh).
#pragma once
#include "libm_match.cuh"

#include <cstdint>
#include <vector>

namespace ngb {
struct HostMathTable {
  std::vector<uint32_t> start; // bucket b: entries [start[b], start[b+1])
  std::vector<uint16_t> entries;
  uint32_t lo = 0, hi = 0;     // input bits covered, [lo, hi)
  int shift = 8, steps = 0;    // bucket size 2^shift; search probes
  // Per exponent of the input: the largest midpoint distance of an entry's
  // formula intermediate, or -1 where there is no entry.
  std::vector<float> skip = std::vector<float>(256, -1.f);
  std::vector<uint32_t> map;   // 3-bit codes of the inputs [map_lo, map_hi), 10 a word (or empty)
  uint32_t map_lo = 0, map_hi = 0;
};
// Built once per process (thread-safe), by evaluating the host library and
// the device formula on every input that can differ.  tanh is keyed by |x|;
// the sigmoid has one table for x >= 0 and one for x < 0, keyed by |x|.
const HostMathTable &tanh_table();
const HostMathTable &sigmoid_table(bool negative);
} // namespace ngb
