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
};
// Built once per process (thread-safe), by evaluating the host library and
// the device formula on every input that can differ.
const HostMathTable &tanh_table();
const HostMathTable &sigmoid_table();
} // namespace ngb
