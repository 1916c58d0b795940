// C++17 adapter: the reference engine's CUDA Linear functions implemented on
// top of the b200 C ABI (include/b200_linear.h).
//
// Drop-in for six definitions in the reference's src/cuda/kernels.cu
// (gemv_bf16 1540-1564, lm_head_bf16 1566-1579, gemm_bf16 1600-1625,
// gemv_w8a16 1627-1655, gemm_w8a16 1657-1684, argmax_bf16 1534-1538; declared
// in include/infer/cuda_ops.hpp:24-55,102-103).  Compile this file against
// the reference tree (it includes "infer/cuda_ops.hpp" from there) and link
// libb200linear.so; the reference's own definitions of these six functions
// are compiled out of kernels.cu (for example by renaming them with -D on
// its compile line).  Signatures, argument meaning and error behaviour
// are the reference's: a failed call throws infer::Error.
//
// `--linear-kernel custom` (the engine default) therefore runs the sm_100a
// kernels.  gemv_bf16_cublas / gemm_bf16_cublas are not replaced: the
// `--linear-kernel cublas` baseline stays the reference's own code.

#include <cstdint>
#include <sstream>
#include <string>

#include "b200_linear.h"
#include "infer/cuda_ops.hpp"

namespace infer::cuda {
namespace {

void check(int status, const char* what) {
  if (status != B200_OK) {
    std::ostringstream os;
    os << what << " failed: " << b200_status_string(status) << " (status "
       << status << ")";
    throw Error(os.str());
  }
}

inline const uint16_t* bits(const __nv_bfloat16* p) {
  return reinterpret_cast<const uint16_t*>(p);
}
inline uint16_t* bits(__nv_bfloat16* p) { return reinterpret_cast<uint16_t*>(p); }

}  // namespace

void gemv_bf16(const __nv_bfloat16* weight, const __nv_bfloat16* bias,
               const __nv_bfloat16* input, __nv_bfloat16* output,
               int out_features, int in_features, cudaStream_t stream) {
  check(b200_gemv_bf16(bits(weight), bits(bias), bits(input), bits(output),
                       out_features, in_features, stream),
        "gemv_bf16");
}

void gemv_w8a16(const int8_t* weight, const __nv_bfloat16* scales,
                int group_size, const __nv_bfloat16* bias,
                const __nv_bfloat16* input, __nv_bfloat16* output,
                int out_features, int in_features, cudaStream_t stream) {
  check(b200_gemv_w8a16(weight, bits(scales), group_size, bits(bias),
                        bits(input), bits(output), out_features, in_features,
                        stream),
        "gemv_w8a16");
}

void gemm_bf16(const __nv_bfloat16* weight, const __nv_bfloat16* bias,
               const __nv_bfloat16* input, __nv_bfloat16* output, int tokens,
               int out_features, int in_features, cudaStream_t stream) {
  check(b200_gemm_bf16(bits(weight), bits(bias), bits(input), bits(output),
                       tokens, out_features, in_features, stream),
        "gemm_bf16");
}

void gemm_w8a16(const int8_t* weight, const __nv_bfloat16* scales,
                int group_size, const __nv_bfloat16* bias,
                const __nv_bfloat16* input, __nv_bfloat16* output, int tokens,
                int out_features, int in_features, cudaStream_t stream) {
  check(b200_gemm_w8a16(weight, bits(scales), group_size, bits(bias),
                        bits(input), bits(output), tokens, out_features,
                        in_features, stream),
        "gemm_w8a16");
}

void lm_head_bf16(const __nv_bfloat16* weight, const __nv_bfloat16* bias,
                  const __nv_bfloat16* input, __nv_bfloat16* logits,
                  float* block_max_value, int* block_max_index, int* argmax,
                  int vocab, int in_features, cudaStream_t stream) {
  check(b200_lm_head_bf16(bits(weight), bits(bias), bits(input), bits(logits),
                          block_max_value, block_max_index, argmax, vocab,
                          in_features, stream),
        "lm_head_bf16");
}

void argmax_bf16(const __nv_bfloat16* values, int n, int* output,
                 cudaStream_t stream) {
  check(b200_argmax_bf16(bits(values), n, output, stream), "argmax_bf16");
}

}  // namespace infer::cuda
