/*
 * ORACLE (test infrastructure only).  The host C library's tanhf and the
 * sigmoid 1 / (1 + expf(-x)) in fp32, exactly as the reference CPU engine
 * evaluates them (src/native/NeuralEngine.cpp:9 sigmoid, :84-85 tanh), over
 * arrays, for checking the device's versions.
 */
#include <math.h>
#include <stddef.h>

void om_libm_eval(const float *x, size_t n, float *tanh_out, float *sigmoid_out) {
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < (long long)n; ++i) {
    if (tanh_out) tanh_out[i] = tanhf(x[i]);
    if (sigmoid_out) sigmoid_out[i] = 1.f / (1.f + expf(-x[i]));
  }
}
