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
                            libm_match::MathTable sp, libm_match::MathTable sn) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  if (tanh_out) tanh_out[i] = libm_match::tanh_host(x[i], tt);
  if (sig_out) sig_out[i] = libm_match::sigmoid_host(x[i], sp, sn);
}

libm_match::MathTable upload(const HostMathTable &h, DeviceBuffer &start, DeviceBuffer &entries, DeviceBuffer &map, DeviceBuffer &skip) {
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
  t.shift = h.shift;
  t.steps = h.steps;
  skip.reset(h.skip.size() * 4);
  NGB_CUDA(cudaMemcpy(skip.as<void>(), h.skip.data(), h.skip.size() * 4, cudaMemcpyHostToDevice));
  t.skip = skip.as<float>();
  if (!h.map.empty()) {
    map.reset(h.map.size() * 4);
    NGB_CUDA(cudaMemcpy(map.as<void>(), h.map.data(), h.map.size() * 4, cudaMemcpyHostToDevice));
    t.map = map.as<uint32_t>();
    t.map_lo = h.map_lo;
    t.map_hi = h.map_hi;
  }
  return t;
}
} // namespace
} // namespace ngb

using namespace ngb;

extern "C" int ng_math_eval(const float *x, size_t n, float *tanh_out, float *sigmoid_out) {
  return guarded([&] {
    if (!x || (!tanh_out && !sigmoid_out)) throw std::invalid_argument("Null input/output");
    require_sm100_device();
    DeviceBuffer ts, te, tm, tk, ps, pe, pm, pk, ns, ne, nm, nk, dx(n * 4 + 4), dt(n * 4 + 4), ds(n * 4 + 4);
    const libm_match::MathTable tt = upload(tanh_table(), ts, te, tm, tk),
                                sp = upload(sigmoid_table(false), ps, pe, pm, pk),
                                sn = upload(sigmoid_table(true), ns, ne, nm, nk);
    NGB_CUDA(cudaMemcpy(dx.as<void>(), x, n * 4, cudaMemcpyHostToDevice));
    for (size_t o = 0; o < n; o += size_t(1) << 30) {
      const int m = int(std::min(n - o, size_t(1) << 30));
      k_math_eval<<<(m + 255) / 256, 256>>>(dx.as<float>() + o, m, tanh_out ? dt.as<float>() + o : nullptr,
                                            sigmoid_out ? ds.as<float>() + o : nullptr, tt, sp, sn);
      NGB_CUDA(cudaGetLastError());
    }
    if (tanh_out) NGB_CUDA(cudaMemcpy(tanh_out, dt.as<void>(), n * 4, cudaMemcpyDeviceToHost));
    if (sigmoid_out) NGB_CUDA(cudaMemcpy(sigmoid_out, ds.as<void>(), n * 4, cudaMemcpyDeviceToHost));
  });
}
