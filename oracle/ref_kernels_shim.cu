// C entry points around the reference's own CUDA Linear functions
// (src/cuda/kernels.cu:1540-1704), which oracle/Makefile compiles unchanged
// from the reference sources for sm_100a.  They are the same-box comparison
// for parity tests on the GPU.  Test infrastructure only; never part of the
// product library.  Each wrapper returns 0, or -1 when the reference throws
// infer::Error (its error behaviour, src/cuda/kernels.cu:1631,1661).
#include "infer/cuda_ops.hpp"

namespace {
template <class F>
int guarded(F&& f) {
  try {
    f();
  } catch (const infer::Error&) {
    return -1;
  } catch (...) {
    return -2;
  }
  return 0;
}
using bf16 = __nv_bfloat16;
}  // namespace

extern "C" {

int ref_gemv_bf16(const void* w, const void* bias, const void* x, void* y,
                  int n, int k, cudaStream_t s) {
  return guarded([&] {
    infer::cuda::gemv_bf16((const bf16*)w, (const bf16*)bias, (const bf16*)x,
                           (bf16*)y, n, k, s);
  });
}

int ref_gemv_w8a16(const void* w, const void* scales, int group,
                   const void* bias, const void* x, void* y, int n, int k,
                   cudaStream_t s) {
  return guarded([&] {
    infer::cuda::gemv_w8a16((const int8_t*)w, (const bf16*)scales, group,
                            (const bf16*)bias, (const bf16*)x, (bf16*)y, n, k,
                            s);
  });
}

int ref_gemm_bf16(const void* w, const void* bias, const void* x, void* y,
                  int m, int n, int k, cudaStream_t s) {
  return guarded([&] {
    infer::cuda::gemm_bf16((const bf16*)w, (const bf16*)bias, (const bf16*)x,
                           (bf16*)y, m, n, k, s);
  });
}

int ref_gemm_w8a16(const void* w, const void* scales, int group,
                   const void* bias, const void* x, void* y, int m, int n,
                   int k, cudaStream_t s) {
  return guarded([&] {
    infer::cuda::gemm_w8a16((const int8_t*)w, (const bf16*)scales, group,
                            (const bf16*)bias, (const bf16*)x, (bf16*)y, m, n,
                            k, s);
  });
}

int ref_lm_head_bf16(const void* w, const void* bias, const void* x,
                     void* logits, float* block_max_value,
                     int* block_max_index, int* argmax, int vocab, int k,
                     cudaStream_t s) {
  return guarded([&] {
    infer::cuda::lm_head_bf16((const bf16*)w, (const bf16*)bias,
                              (const bf16*)x, (bf16*)logits, block_max_value,
                              block_max_index, argmax, vocab, k, s);
  });
}

int ref_argmax_bf16(const void* values, int n, int* out, cudaStream_t s) {
  return guarded(
      [&] { infer::cuda::argmax_bf16((const bf16*)values, n, out, s); });
}

}  // extern "C"
