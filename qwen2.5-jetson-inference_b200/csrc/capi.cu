// extern "C" boundary (include/b200_linear.h): argument validation and
// dispatch to the kernels.  Error behaviour mirrors the reference functions
// (src/cuda/kernels.cu:1540-1704), which throw infer::Error; here the same
// conditions return a negative status instead, and launch failures return
// the cudaError_t.
#include "b200_linear.h"
#include "kernels.h"

namespace b200 {
cudaError_t read_device_status(int* value, bool clear);  // gemm_sm100.cu
cudaError_t read_gemv_status(int* value, bool clear);    // gemv.cu
cudaError_t read_comm_status(int* value, bool clear);    // sharded.cu
cudaError_t read_w8t_status(int* value, bool clear);     // gemm_w8t.cu
cudaError_t read_i8tc_status(int* value, bool clear);    // gemv_i8tc.cu
cudaError_t read_att_status(int* value, bool clear);     // attention_tc.cu
}

using b200::bf16;

namespace {

inline int status_of(cudaError_t e) { return e == cudaSuccess ? B200_OK : int(e); }

inline const bf16* as_bf16(const uint16_t* p) {
  return reinterpret_cast<const bf16*>(p);
}
inline bf16* as_bf16(uint16_t* p) { return reinterpret_cast<bf16*>(p); }

int check_linear_args(const void* weight, const void* input,
                      const void* output, int tokens, int out_features,
                      int in_features) {
  if (tokens < 0 || out_features < 0 || in_features < 0) {
    return B200_ERR_INVALID_ARGUMENT;
  }
  if (tokens == 0 || out_features == 0) return B200_OK;
  if (output == nullptr) return B200_ERR_INVALID_ARGUMENT;
  if (in_features > 0 && (weight == nullptr || input == nullptr)) {
    return B200_ERR_INVALID_ARGUMENT;
  }
  return B200_OK;
}

int gemm_common(bool w8, const void* weight, const uint16_t* scales,
                const uint16_t* bias, const uint16_t* input, uint16_t* output,
                int tokens, int out_features, int in_features,
                cudaStream_t stream) {
  int rc = check_linear_args(weight, input, output, tokens, out_features,
                             in_features);
  if (rc != B200_OK) return rc;
  if (tokens == 0 || out_features == 0) return B200_OK;
  if (w8 && in_features > 0 && scales == nullptr) return B200_ERR_INVALID_ARGUMENT;
  if (tokens == 1) {
    // One token: the weight stream kernel is the right tool (the reference's
    // m=1 prefill falls to its slow bounds-checked path instead).
    return status_of(b200::launch_gemv(w8, weight, as_bf16(scales),
                                       as_bf16(bias), as_bf16(input),
                                       as_bf16(output), out_features,
                                       in_features, nullptr, nullptr, stream,
                                       nullptr));
  }
  if (b200::gemm_tc_supported(w8, weight, input, output, tokens, out_features,
                              in_features)) {
    return status_of(b200::launch_gemm_tc(w8, weight, as_bf16(scales),
                                          as_bf16(bias), as_bf16(input),
                                          as_bf16(output), tokens,
                                          out_features, in_features, stream));
  }
  return status_of(b200::launch_gemm_simt(w8, weight, as_bf16(scales),
                                          as_bf16(bias), as_bf16(input),
                                          as_bf16(output), tokens,
                                          out_features, in_features, stream));
}

int lm_head_common(bool w8, const void* weight, const uint16_t* scales,
                   const uint16_t* bias, const uint16_t* input,
                   uint16_t* logits, float* block_max_value,
                   int* block_max_index, int* argmax, int vocab,
                   int in_features, cudaStream_t stream) {
  if (vocab < 0 || in_features < 0) return B200_ERR_INVALID_ARGUMENT;
  if (argmax == nullptr) return B200_ERR_INVALID_ARGUMENT;
  if (vocab == 0) {
    return status_of(cudaMemsetAsync(argmax, 0, sizeof(int), stream));
  }
  if (logits == nullptr) return B200_ERR_INVALID_ARGUMENT;
  if (block_max_value == nullptr || block_max_index == nullptr) {
    return B200_ERR_WORKSPACE;
  }
  if (in_features > 0 && (weight == nullptr || input == nullptr)) {
    return B200_ERR_INVALID_ARGUMENT;
  }
  if (w8 && in_features > 0 && scales == nullptr) return B200_ERR_INVALID_ARGUMENT;
  int grid = 0;
  cudaError_t e = b200::launch_gemv(w8, weight, as_bf16(scales), as_bf16(bias),
                                    as_bf16(input), as_bf16(logits), vocab,
                                    in_features, block_max_value,
                                    block_max_index, stream, &grid);
  if (e != cudaSuccess) return int(e);
  // Every launch shape uses >= 8 rows per CTA, so grid <= ceil(vocab / 8),
  // the workspace the reference engine allocates.
  if (grid > (vocab + 7) / 8) return B200_ERR_WORKSPACE;
  return status_of(b200::launch_argmax_partials(block_max_value,
                                                block_max_index, grid, argmax,
                                                stream));
}

}  // namespace

extern "C" {

int b200_version(void) { return 200; }

int b200_set_summation_order(int order) {
  if (order != B200_ORDER_FAST && order != B200_ORDER_REFERENCE) {
    return B200_ERR_INVALID_ARGUMENT;
  }
  b200::set_summation_order(order);
  return B200_OK;
}

int b200_summation_order(void) { return b200::summation_order(); }

const char* b200_status_string(int status) {
  switch (status) {
    case B200_OK: return "ok";
    case B200_ERR_INVALID_ARGUMENT: return "invalid argument (null pointer or negative size)";
    case B200_ERR_GROUP_SIZE: return "w8a16 group size must be 64";
    case B200_ERR_WORKSPACE: return "workspace missing or too small";
    case B200_ERR_TOO_LARGE: return "size exceeds the supported maximum";
    case B200_ERR_NCCL: return "NCCL call failed";
    default: break;
  }
  if (status > 0) return cudaGetErrorString(static_cast<cudaError_t>(status));
  return "unknown status";
}

int b200_device_status(int clear) {
  int gemm = 0, gemv = 0, comm = 0, w8t = 0;
  cudaError_t e = b200::read_device_status(&gemm, clear != 0);  // synchronises
  if (e == cudaSuccess) e = b200::read_gemv_status(&gemv, clear != 0);
  if (e == cudaSuccess) e = b200::read_comm_status(&comm, clear != 0);
  int i8 = 0;
  if (e == cudaSuccess) e = b200::read_w8t_status(&w8t, clear != 0);
  if (e == cudaSuccess) e = b200::read_i8tc_status(&i8, clear != 0);
  int att = 0;
  if (e == cudaSuccess) e = b200::read_att_status(&att, clear != 0);
  if (e != cudaSuccess) return -int(e);
  return gemm != 0 ? gemm : gemv != 0 ? gemv : comm != 0 ? comm : w8t != 0 ? w8t : i8 != 0 ? i8
                                                                                         : att;
}

int b200_gemv_bf16(const uint16_t* weight, const uint16_t* bias,
                   const uint16_t* input, uint16_t* output, int out_features,
                   int in_features, b200_stream_t stream) {
  int rc = check_linear_args(weight, input, output, 1, out_features,
                             in_features);
  if (rc != B200_OK || out_features == 0) return rc;
  return status_of(b200::launch_gemv(false, weight, nullptr, as_bf16(bias),
                                     as_bf16(input), as_bf16(output),
                                     out_features, in_features, nullptr,
                                     nullptr, stream, nullptr));
}

int b200_gemv_w8a16(const int8_t* weight, const uint16_t* scales,
                    int group_size, const uint16_t* bias,
                    const uint16_t* input, uint16_t* output, int out_features,
                    int in_features, b200_stream_t stream) {
  if (group_size != 64) return B200_ERR_GROUP_SIZE;
  int rc = check_linear_args(weight, input, output, 1, out_features,
                             in_features);
  if (rc != B200_OK || out_features == 0) return rc;
  if (in_features > 0 && scales == nullptr) return B200_ERR_INVALID_ARGUMENT;
  return status_of(b200::launch_gemv(true, weight, as_bf16(scales),
                                     as_bf16(bias), as_bf16(input),
                                     as_bf16(output), out_features,
                                     in_features, nullptr, nullptr, stream,
                                     nullptr));
}

int b200_gemm_reserve_scratch(size_t bytes) {
  return status_of(b200::reserve_gemm_scratch(bytes));
}

int b200_gemm_bf16(const uint16_t* weight, const uint16_t* bias,
                   const uint16_t* input, uint16_t* output, int tokens,
                   int out_features, int in_features, b200_stream_t stream) {
  return gemm_common(false, weight, nullptr, bias, input, output, tokens,
                     out_features, in_features, stream);
}

int b200_gemm_w8a16(const int8_t* weight, const uint16_t* scales,
                    int group_size, const uint16_t* bias,
                    const uint16_t* input, uint16_t* output, int tokens,
                    int out_features, int in_features, b200_stream_t stream) {
  if (group_size != 64) return B200_ERR_GROUP_SIZE;
  return gemm_common(true, weight, scales, bias, input, output, tokens,
                     out_features, in_features, stream);
}

size_t b200_lm_head_workspace_bytes(int vocab, int in_features) {
  (void)in_features;
  if (vocab <= 0) return 0;
  const size_t blocks = (size_t(vocab) + 7) / 8;
  return blocks * (sizeof(float) + sizeof(int));
}

int b200_lm_head_bf16(const uint16_t* weight, const uint16_t* bias,
                      const uint16_t* input, uint16_t* logits,
                      float* block_max_value, int* block_max_index,
                      int* argmax, int vocab, int in_features,
                      b200_stream_t stream) {
  return lm_head_common(false, weight, nullptr, bias, input, logits,
                        block_max_value, block_max_index, argmax, vocab,
                        in_features, stream);
}

int b200_lm_head_w8a16(const int8_t* weight, const uint16_t* scales,
                       int group_size, const uint16_t* bias,
                       const uint16_t* input, uint16_t* logits,
                       float* block_max_value, int* block_max_index,
                       int* argmax, int vocab, int in_features,
                       b200_stream_t stream) {
  if (group_size != 64) return B200_ERR_GROUP_SIZE;
  return lm_head_common(true, weight, scales, bias, input, logits,
                        block_max_value, block_max_index, argmax, vocab,
                        in_features, stream);
}

int b200_argmax_bf16(const uint16_t* values, int n, int* output,
                     b200_stream_t stream) {
  if (output == nullptr) return B200_ERR_INVALID_ARGUMENT;
  if (n > 0 && values == nullptr) return B200_ERR_INVALID_ARGUMENT;
  return status_of(b200::launch_argmax_bf16(as_bf16(values), n < 0 ? 0 : n,
                                            output, stream));
}

}  // extern "C"

extern "C" {

size_t b200_w8a16_packed_bytes(int out_features, int in_features) {
  return b200::w8a16_packed_bytes(out_features, in_features);
}

int b200_pack_w8a16(const int8_t* weight, int out_features, int in_features, void* packed,
                    b200_stream_t stream) {
  if (out_features < 0 || in_features < 0) return B200_ERR_INVALID_ARGUMENT;
  if (out_features == 0 || in_features == 0) return B200_OK;
  if (weight == nullptr || packed == nullptr || in_features % 16 != 0 ||
      (reinterpret_cast<uintptr_t>(weight) & 15u) != 0 ||
      (reinterpret_cast<uintptr_t>(packed) & 15u) != 0) {
    return B200_ERR_INVALID_ARGUMENT;
  }
  return status_of(b200::launch_pack_w8a16(weight, out_features, in_features, packed,
                                           static_cast<cudaStream_t>(stream)));
}

int b200_gemm_w8a16_packed(const void* packed, const uint16_t* scales, int group_size,
                           const uint16_t* bias, const uint16_t* input, uint16_t* output,
                           int tokens, int out_features, int in_features,
                           b200_stream_t stream) {
  if (group_size != 64) return B200_ERR_GROUP_SIZE;
  int rc = check_linear_args(packed, input, output, tokens, out_features, in_features);
  if (rc != B200_OK) return rc;
  if (tokens == 0 || out_features == 0) return B200_OK;
  if (in_features == 0 || scales == nullptr || in_features % 16 != 0 ||
      (reinterpret_cast<uintptr_t>(packed) & 15u) != 0 ||
      (reinterpret_cast<uintptr_t>(input) & 15u) != 0) {
    return B200_ERR_INVALID_ARGUMENT;
  }
  return status_of(b200::launch_gemm_w8t(packed, as_bf16(scales), as_bf16(bias),
                                         as_bf16(input), as_bf16(output), tokens,
                                         out_features, in_features, out_features,
                                         static_cast<cudaStream_t>(stream), packed));
}

}  // extern "C"
