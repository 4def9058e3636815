// ng_math_eval: the tick kernels' sigmoid and tanh on caller inputs, for
// checking them against the host C library (libm_match.cuh).
#include "capi_common.h"
#include "common.h"
#include "math_tables.h"
#include "neurogen_b200.h"

#include <cuda_runtime.h>

#include <algorithm>

namespace ngb {
namespace {
__global__ void k_math_eval(const float *x, int n, float *tanh_out, float *sig_out, libm_match::MathTable tt,
                            libm_match::MathTable st) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  if (tanh_out) tanh_out[i] = libm_match::tanh_host(x[i], tt);
  if (sig_out) sig_out[i] = libm_match::sigmoid_host(x[i], st);
}

libm_match::MathTable upload(const HostMathTable &h, DeviceBuffer &start, DeviceBuffer &entries) {
  start.reset(h.start.size() * 4);
  entries.reset((h.entries.size() + 1) * 2);
  NGB_CUDA(cudaMemcpy(start.as<void>(), h.start.data(), h.start.size() * 4, cudaMemcpyHostToDevice));
  if (!h.entries.empty())
    NGB_CUDA(cudaMemcpy(entries.as<void>(), h.entries.data(), h.entries.size() * 2, cudaMemcpyHostToDevice));
  libm_match::MathTable t;
  t.start = start.as<uint32_t>();
  t.entries = entries.as<uint16_t>();
  t.lo = h.lo;
  t.hi = h.hi;
  return t;
}
} // namespace
} // namespace ngb

using namespace ngb;

extern "C" int ng_math_eval(const float *x, size_t n, float *tanh_out, float *sigmoid_out) {
  return guarded([&] {
    if (!x || (!tanh_out && !sigmoid_out)) throw std::invalid_argument("Null input/output");
    require_sm100_device();
    DeviceBuffer ts, te, ss, se, dx(n * 4 + 4), dt(n * 4 + 4), ds(n * 4 + 4);
    const libm_match::MathTable tt = upload(tanh_table(), ts, te), st = upload(sigmoid_table(), ss, se);
    NGB_CUDA(cudaMemcpy(dx.as<void>(), x, n * 4, cudaMemcpyHostToDevice));
    for (size_t o = 0; o < n; o += size_t(1) << 30) {
      const int m = int(std::min(n - o, size_t(1) << 30));
      k_math_eval<<<(m + 255) / 256, 256>>>(dx.as<float>() + o, m, tanh_out ? dt.as<float>() + o : nullptr,
                                            sigmoid_out ? ds.as<float>() + o : nullptr, tt, st);
      NGB_CUDA(cudaGetLastError());
    }
    if (tanh_out) NGB_CUDA(cudaMemcpy(tanh_out, dt.as<void>(), n * 4, cudaMemcpyDeviceToHost));
    if (sigmoid_out) NGB_CUDA(cudaMemcpy(sigmoid_out, ds.as<void>(), n * 4, cudaMemcpyDeviceToHost));
  });
}
