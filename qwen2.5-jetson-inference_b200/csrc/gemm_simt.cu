// CUDA-core GEMM for shapes the tensor-core path does not take (in_features
// not a multiple of 8, unaligned pointers).  Same arithmetic contract as the
// tensor-core path: FP32 accumulation, W8A16 weights dequantised to
// bf16(q * s) first (reference src/cuda/kernels.cu:1075-1094), bias added to
// the FP32 sum, BF16 round-to-nearest-even output.  The reference's own
// fallback for these shapes is linear_w8a16_kernel / gemm_bf16_wmma_kernel
// (src/cuda/kernels.cu:605-708, 1324-1387).
#include "common.cuh"
#include "kernels.h"

namespace b200 {
namespace {

constexpr int kTile = 64;
constexpr int kStepK = 16;

template <bool kW8>
__global__ void __launch_bounds__(256)
gemm_simt_kernel(const void* __restrict__ weight,
                 const bf16* __restrict__ scales, const bf16* __restrict__ bias,
                 const bf16* __restrict__ input, bf16* __restrict__ output,
                 int m, int n, int k) {
  __shared__ float xs[kStepK][kTile + 1];
  __shared__ float ws[kStepK][kTile + 1];
  const int m0 = blockIdx.y * kTile;
  const int n0 = blockIdx.x * kTile;
  const int tx = threadIdx.x % 16;  // n direction
  const int ty = threadIdx.x / 16;  // m direction
  const int groups = (k + 63) / 64;
  float acc[4][4] = {};
  pdl_wait_primary();
  for (int k0 = 0; k0 < k; k0 += kStepK) {
    for (int i = threadIdx.x; i < kTile * kStepK; i += 256) {
      const int row = i / kStepK;
      const int kk = i % kStepK;
      const int gk = k0 + kk;
      const int gm = m0 + row;
      const int gn = n0 + row;
      xs[kk][row] = (gm < m && gk < k)
                        ? __bfloat162float(input[size_t(gm) * k + gk])
                        : 0.0f;
      float wv = 0.0f;
      if (gn < n && gk < k) {
        if constexpr (kW8) {
          const int8_t q = static_cast<const int8_t*>(weight)[size_t(gn) * k + gk];
          const float s = __bfloat162float(scales[size_t(gn) * groups + gk / 64]);
          wv = __bfloat162float(__float2bfloat16_rn(float(q) * s));
        } else {
          wv = __bfloat162float(static_cast<const bf16*>(weight)[size_t(gn) * k + gk]);
        }
      }
      ws[kk][row] = wv;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kStepK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = xs[kk][ty + 16 * i];
        b[i] = ws[kk][tx + 16 * i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gm = m0 + ty + 16 * i;
    if (gm >= m) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gn = n0 + tx + 16 * j;
      if (gn >= n) continue;
      const float b = bias ? __bfloat162float(bias[gn]) : 0.0f;
      output[size_t(gm) * n + gn] = __float2bfloat16_rn(acc[i][j] + b);
    }
  }
}

}  // namespace

cudaError_t launch_gemm_simt(bool w8, const void* weight, const bf16* scales,
                             const bf16* bias, const bf16* input, bf16* output,
                             int m, int n, int k, cudaStream_t stream) {
  if (m <= 0 || n <= 0) return cudaSuccess;
  const dim3 grid((n + kTile - 1) / kTile, (m + kTile - 1) / kTile);
  if (grid.y > 65535) return cudaErrorInvalidConfiguration;
  if (w8) {
    gemm_simt_kernel<true><<<grid, 256, 0, stream>>>(weight, scales, bias,
                                                     input, output, m, n, k);
  } else {
    gemm_simt_kernel<false><<<grid, 256, 0, stream>>>(weight, scales, bias,
                                                      input, output, m, n, k);
  }
  return cudaGetLastError();
}

}  // namespace b200
