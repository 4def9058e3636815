// Shared host-side helpers of the B200 engine: CUDA error checks that turn
// failures into C++ exceptions (the C ABI converts those to -1 / NULL plus an
// ng_error() message, like src/native/NeuralEngine.cpp:193-267), and a small
// owning device buffer.
#pragma once
#include <cuda_runtime.h>
#include <cstddef>
#include <stdexcept>
#include <string>
#include <utility>

namespace ngb {

inline void cuda_check(cudaError_t r, const char *what) {
  if (r != cudaSuccess)
    throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(r));
}
#define NGB_CUDA(call) ::ngb::cuda_check((call), #call)

// Owning device allocation (bytes); moves, never copies.
class DeviceBuffer {
public:
  DeviceBuffer() = default;
  explicit DeviceBuffer(size_t bytes) { reset(bytes); }
  DeviceBuffer(const DeviceBuffer &) = delete;
  DeviceBuffer &operator=(const DeviceBuffer &) = delete;
  DeviceBuffer(DeviceBuffer &&o) noexcept : p_(std::exchange(o.p_, nullptr)), n_(std::exchange(o.n_, 0)) {}
  DeviceBuffer &operator=(DeviceBuffer &&o) noexcept {
    if (this != &o) {
      release();
      p_ = std::exchange(o.p_, nullptr);
      n_ = std::exchange(o.n_, 0);
    }
    return *this;
  }
  ~DeviceBuffer() { release(); }
  void reset(size_t bytes) {
    release();
    if (bytes) NGB_CUDA(cudaMalloc(&p_, bytes));
    n_ = bytes;
  }
  template <class T> T *as() const { return static_cast<T *>(p_); }
  size_t bytes() const { return n_; }

private:
  void release() {
    if (p_) cudaFree(p_);
    p_ = nullptr;
    n_ = 0;
  }
  void *p_ = nullptr;
  size_t n_ = 0;
};

// Throws unless the current device is a Blackwell datacenter part (sm_100):
// the kernels are compiled for sm_100a only and nothing else may run them.
int require_sm100_device();
std::string device_label(int device);

} // namespace ngb
