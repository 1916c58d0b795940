// Internal launch interface between the C ABI (capi.cu) and the kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace b200 {

using bf16 = __nv_bfloat16;

// Optional fusions of the decode GEMV, used by the native decode engine
// (engine.cu) to fold the layers around a Linear into its load and store:
//   in_mode 1: x' = bf16(x * w * rsqrt(mean(x^2) + eps)) (RMSNorm of the
//              input, reference src/cuda/kernels.cu:64-116);
//   in_mode 2: the input holds [gate | up] (2 x in_features) and
//              x' = bf16(silu(gate) * up) (reference kernels.cu:302-324);
//   residual:  residual[n] = bf16(residual[n] + bf16(y[n])) replaces the
//              output store (reference add_inplace_bf16, kernels.cu:285-300).
struct GemvFusion {
  int in_mode = 0;
  const bf16* norm_w = nullptr;
  float eps = 0.0f;
  bf16* residual = nullptr;
};

// gemv.cu
// Summation order of the decode GEMV / LM head (B200_ORDER_FAST or
// B200_ORDER_REFERENCE); process-wide, initialised from the environment
// variable B200_SUMMATION_ORDER ("reference" or "fast").
int summation_order();
void set_summation_order(int order);
bool gemv_uses_fast_path(bool w8, const void* weight, const void* input,
                         int k);
// CTA count launch_gemv will use for these arguments (lm_head: the form with
// argmax partials), without launching anything; 0 when n <= 0.
int gemv_grid(bool w8, const void* weight, const bf16* scales,
              const void* input, int n, int k, bool lm_head);
// Launches the GEMV (block_value == nullptr) or the LM-head GEMV with
// per-CTA argmax partials; *grid_out receives the CTA count.
cudaError_t launch_gemv(bool w8, const void* weight, const bf16* scales,
                        const bf16* bias, const bf16* input, bf16* output,
                        int n, int k, float* block_value, int* block_index,
                        cudaStream_t stream, int* grid_out,
                        const GemvFusion* fusion = nullptr);
cudaError_t launch_argmax_partials(const float* block_value,
                                   const int* block_index, int count,
                                   int* argmax, cudaStream_t stream);
cudaError_t launch_argmax_bf16(const bf16* values, int n, int* out,
                               cudaStream_t stream);

// gemv_i8tc.cu: W8A16 GEMV on the integer tensor cores (k % 64 == 0,
// 64 <= k <= 6144, 16-byte aligned weight and input).
bool gemv_i8tc_supported(const void* weight, const void* input, const void* scales, int n,
                         int k);
int gemv_i8tc_grid(int n);
cudaError_t launch_gemv_i8tc(const void* weight, const bf16* scales, const bf16* bias,
                             const bf16* input, bf16* output, int n, int k, float* block_value,
                             int* block_index, cudaStream_t stream, int* grid_out);

// attention_tc.cu: causal GQA prefill attention on the tensor cores
// (head_dim 64): q rows [tokens][q_stride] (head h at column h*64), caches
// [kv_heads][max_seq][64], query t at position pos0 + t attends [0, pos0+t].
cudaError_t launch_attention_prefill_tc(const bf16* q, int q_stride, const bf16* kcache,
                                        const bf16* vcache, bf16* out, int out_stride, int tokens,
                                        int pos0, int heads, int kv_heads, int max_seq,
                                        cudaStream_t stream);

// gemm_simt.cu: any shape / alignment, CUDA cores.
cudaError_t launch_gemm_simt(bool w8, const void* weight, const bf16* scales,
                             const bf16* bias, const bf16* input, bf16* output,
                             int m, int n, int k, cudaStream_t stream);

// Extra destinations of a GEMM's output tiles: the same tile is stored at
// out + delta[i] bytes for each i < n (the output buffers of the other GPUs
// of a node, mapped into this process), with plain 16-byte stores.
struct PeerOuts {
  long long delta[7] = {0, 0, 0, 0, 0, 0, 0};
  int n = 0;
};

// gemm_sm100.cu: tcgen05 + TMA + TMEM path.
bool gemm_tc_supported(bool w8, const void* weight, const void* input,
                       const void* output, int m, int n, int k);
cudaError_t launch_gemm_tc(bool w8, const void* weight, const bf16* scales,
                           const bf16* bias, const bf16* input, bf16* output,
                           int m, int n, int k, cudaStream_t stream);
// Same with an output row stride (ldc, elements) and peer destinations.
cudaError_t launch_gemm_tc_peers(bool w8, const void* weight, const bf16* scales,
                                 const bf16* bias, const bf16* input, bf16* output,
                                 int m, int n, int k, int ldc, const PeerOuts& peers,
                                 cudaStream_t stream);

// gemm_w8t.cu: W8A16 GEMM with the dequantised weight tiles in TMEM
// (computes Y^T = W . X^T; any m, n; k % 16 == 0, 16-byte aligned W and X).
bool gemm_w8t_supported(const void* weight, const void* input, const void* output, int m,
                        int n, int k);
cudaError_t launch_gemm_w8t(const void* weight, const bf16* scales, const bf16* bias,
                            const bf16* input, bf16* output, int m, int n, int k, int ldc,
                            cudaStream_t stream, const void* packed = nullptr);
// Pre-packed W8A16 weights (tile-major 16 KB blocks in the kernels'
// shared-memory layout); `packed` given to launch_gemm_w8t replaces the
// strided TMA weight loads by 1-D bulk copies.
// K split across a thread-block cluster with a fixed-order reduction in
// distributed shared memory (fast summation order; cudaErrorNotSupported for
// shapes it does not take).
cudaError_t launch_gemm_cluster_split(bool w8, const void* weight, const bf16* scales,
                                      const bf16* bias, const bf16* input, bf16* output,
                                      int m, int n, int k, int ldc, cudaStream_t stream);
size_t w8a16_packed_bytes(int n, int k);
cudaError_t launch_pack_w8a16(const int8_t* q, int n, int k, void* packed, cudaStream_t stream);
// The same transposed form with BF16 weights read by the MMA from shared
// memory (same support conditions), for prompts of <= 128 tokens.
cudaError_t launch_gemm_w16t(const bf16* weight, const bf16* bias, const bf16* input,
                             bf16* output, int m, int n, int k, int ldc, cudaStream_t stream);

// Allocates (once per device) the BF16 weight buffer of the two-pass W8A16
// prefill path; bytes == 0 means the default cap.
cudaError_t reserve_gemm_scratch(size_t bytes);

}  // namespace b200
