// C entry points around the reference's CPU FP32 Linear ops
// (src/cpu_ops.cpp:23-30 linear_fp32, :108-123 linear_fp32_batch), compiled
// from the reference sources in place by oracle/Makefile.  Test and
// CPU-baseline infrastructure only; never part of the product library.
#include "infer/cpu_ops.hpp"
#include "cblas.h"

extern "C" {

int ref_cpu_linear_fp32(const float* weight, const float* bias,
                        const float* input, float* output, int out_features,
                        int in_features) {
  try {
    infer::cpu::linear_fp32(weight, bias, input, output, out_features,
                            in_features);
  } catch (...) {
    return -1;
  }
  return 0;
}

int ref_cpu_linear_fp32_batch(const float* weight, const float* bias,
                              const float* input, float* output, int tokens,
                              int out_features, int in_features) {
  try {
    infer::cpu::linear_fp32_batch(weight, bias, input, output, tokens,
                                  out_features, in_features);
  } catch (...) {
    return -1;
  }
  return 0;
}

int ref_cpu_argmax(const float* values, int n) {
  return infer::cpu::argmax(values, n);
}

void ref_cpu_set_threads(int n) { openblas_set_num_threads(n); }
int ref_cpu_get_threads(void) { return openblas_get_num_threads(); }

}  // extern "C"
