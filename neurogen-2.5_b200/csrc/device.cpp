// Device discovery: the engine runs only on sm_100 (B200-class) GPUs.
#include "common.h"

#include <string>

namespace ngb {

int require_sm100_device() {
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || count == 0)
    throw std::runtime_error(std::string("No CUDA device available for the B200 engine (") +
                             (e != cudaSuccess ? cudaGetErrorString(e) : "0 devices") +
                             "); there is no CPU fallback");
  int dev = 0;
  NGB_CUDA(cudaGetDevice(&dev));
  cudaDeviceProp p{};
  NGB_CUDA(cudaGetDeviceProperties(&p, dev));
  if (p.major != 10 || p.minor != 0)
    throw std::runtime_error(std::string("The B200 engine needs an sm_100 GPU; device ") +
                             std::to_string(dev) + " is " + p.name + " (sm_" + std::to_string(p.major) +
                             std::to_string(p.minor) + "); there is no fallback");
  return dev;
}

std::string device_label(int device) {
  cudaDeviceProp p{};
  NGB_CUDA(cudaGetDeviceProperties(&p, device));
  return std::string("cuda: ") + p.name + " (sm_100a)";
}

} // namespace ngb
