// W8A16 decode GEMV (M = 1) on the INTEGER tensor cores.
//
//   y[n] = bf16( sum_g s[n,g] * sum_{k in g} q[n,k] * x[k] + b[n] )
//
// The CUDA-core GEMV spends ~3 instructions per weight byte turning int8
// into float, which caps it below the HBM rate.  Here no CUDA core touches a
// weight byte: the INT8 weights go by TMA into shared memory and straight
// into tcgen05.mma.kind::i8 against an exact integer form of x.
//
// x as integers: for each quantisation group g of 64 values, E_g is the
// largest BF16 exponent in the group and every x_k is written as
// L_k * 2^(E_g - 147) with |L_k| < 2^21 (exact unless an element is more
// than 2^13 below the group's largest, where the dropped bits are below
// 2^-20 of it).  |L_k| splits into three 7-bit limbs l_0 + 128 l_1 +
// 16384 l_2 carrying the sign, each an int8: the B operand is [16 rows =
// limbs (3 used) x K] int8.  One MMA group (two K=32 MMAs, M = 128 weight
// rows, N = 16) gives D[row, limb] = sum_{k in g} q[row,k] * l_limb[k] in
// INT32, exact (|D| < 64 * 127 * 127).  The epilogue adds, per row and
// group, s * 2^(E_g-147) * (D0 + 128 D1 + 16384 D2) to an FP32 sum.
//
// Differences from the CUDA-core GEMV: each group's dot product is exact;
// rounding happens only in the per-group combination, so outputs agree with
// an FP32 restatement to within its own rounding (one BF16 ulp at most).
// The reference-order mode never takes this kernel.
//
// Roles (one persistent CTA per SM, 128-row tiles round robin):
//   all threads  build the limb tile of x for all of K in shared memory
//                (after griddepcontrol.wait; the first weight stages are in
//                flight before it, since weights never depend on it);
//   warp 0       TMA producer: W tiles [128 rows x 128 K] int8, 128-byte
//                swizzle, into a ring of stages;
//   warp 1       TMEM allocator and MMA issuer: per 64-K group two MMAs into
//                16 TMEM columns; 8 groups (4 stages) form a chunk, handed
//                over with one commit (a 4-deep ring of 128-column chunks);
//   warps 4..7   epilogue: thread = weight row; per chunk eight tcgen05.ld,
//                one wait, release, combine; then bias, BF16, store, argmax.
// Every wait is bounded and reports B200_DEVICE_TIMEOUT_PIPELINE.

#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cfloat>
#include <climits>

#include "common.cuh"
#include "gemv_math.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace b200 {

__device__ int g_i8tc_status = 0;

cudaError_t read_i8tc_status(int* value, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(value, g_i8tc_status, sizeof(int));
  if (e != cudaSuccess || !clear) return e;
  const int zero = 0;
  return cudaMemcpyToSymbol(g_i8tc_status, &zero, sizeof(int));
}

bool encode_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                    int elem_bytes, int inner, int outer, int box_inner, int box_outer,
                    CUtensorMapSwizzle swizzle);

namespace {

constexpr int kTileRows = 128;
constexpr int kKB = 128;          // K per stage (two quantisation groups)
constexpr int kStageBytes = kTileRows * kKB;   // 16 KB
constexpr int kMaxStages = 6;   // ring depth (measured: 12 stages ran slower)
constexpr int kLimbRows = 16;     // MMA N (limbs 0..2 used)
constexpr int kLimbBlock = kLimbRows * kKB;    // 2 KB per k-block
constexpr int kChunkGroups = 8;   // groups handed to the epilogue at once
constexpr int kChunkCols = kChunkGroups * 16;  // a group's D = 16 columns
constexpr int kChunks = 4;        // TMEM chunk buffers (4 x 128 = 512 columns)
constexpr int kThreads = 256;
constexpr int kMaxK = 5120;      // limb tile + scale tiles + ring within shared memory
constexpr int kMinRows = 4 * 148 * kTileRows;

// Instruction descriptor, kind::i8: D = S32, A = B = S8, both K-major.
constexpr uint32_t idesc_i8(int m, int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | (uint32_t(n >> 3) << 17) |
         (uint32_t(m >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ bool wait_i(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  return mbar_wait_bounded(bar, parity, abort_flag, B200_DEVICE_TIMEOUT_PIPELINE,
                           &g_i8tc_status);
}

// Byte offset of (row r, column c) in a [rows x 128] tile with the 128-byte
// swizzle (16-byte chunk c/16 of row r at chunk (c/16) ^ (r & 7)).
__device__ __forceinline__ int sw128(int r, int c) {
  return r * 128 + ((((c >> 4) ^ (r & 7))) << 4) + (c & 15);
}

__global__ void __launch_bounds__(kThreads, 1)
gemv_i8tc_kernel(const __grid_constant__ CUtensorMap tmap_w, const uint16_t* __restrict__ scales,
                 const bf16* __restrict__ bias, const bf16* __restrict__ input,
                 bf16* __restrict__ output, int n_rows, int k, float* __restrict__ block_value,
                 int* __restrict__ block_index, const int kStages) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int num_kb = (k + kKB - 1) / kKB;
  const int groups = k / 64;
  unsigned char* ring = smem;
  unsigned char* limbs = ring + kStages * kStageBytes;             // num_kb x 2 KB
  // Two tiles' scales [128 rows x groups] BF16, each one contiguous range of
  // the scale array (rows of a tile are consecutive).
  const int stile_bytes = kTileRows * groups * 2;
  unsigned char* stiles = limbs + num_kb * kLimbBlock;
  float* gfac = reinterpret_cast<float*>(stiles + 2 * stile_bytes);  // [groups]
  uint64_t* bars = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(gfac + groups) + 15) & ~uintptr_t(15));
  const uint32_t bar_full = smem_u32(bars);
  const uint32_t bar_empty = bar_full + 8 * kMaxStages;
  const uint32_t bar_dfull = bar_empty + 8 * kMaxStages;
  const uint32_t bar_dempty = bar_dfull + 8 * kChunks;
  const uint32_t bar_sfull = bar_dempty + 8 * kChunks;
  const uint32_t bar_sempty = bar_sfull + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kMaxStages + 2 * kChunks + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* red_v = reinterpret_cast<float*>(tmem_slot + 2);
  int* red_i = reinterpret_cast<int*>(red_v + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_tiles = (n_rows + kTileRows - 1) / kTileRows;

  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    for (int d = 0; d < kChunks; ++d) {
      mbar_init(bar_dfull + 8 * d, 1);
      mbar_init(bar_dempty + 8 * d, 4);  // one arrival per epilogue warp
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar_sfull + 8 * b, 1);
      mbar_init(bar_sempty + 8 * b, 4);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kChunks * kChunkCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // The weights do not depend on the previous kernel: the first stages are
  // requested before griddepcontrol.wait.
  const int total_steps = ((num_tiles - int(blockIdx.x) + int(gridDim.x) - 1) / int(gridDim.x)) *
                          num_kb;
  // Steps issued before griddepcontrol.wait: none of them may wait (the
  // consumers have not started), so at most one ring's worth and at most the
  // two tiles whose scale buffers are free.
  int first = total_steps < kStages ? total_steps : kStages;
  if (first > 2 * num_kb) first = 2 * num_kb;
  // Step i = k-block i % num_kb of this CTA's tile i / num_kb.  A tile's
  // first step also brings its scales (bulk copy into buffer (i/num_kb) & 1).
  auto issue = [&](int i) -> bool {
    const int ti = i / num_kb, kb = i % num_kb;
    const int tile = int(blockIdx.x) + ti * int(gridDim.x);
    const int s = i % kStages;
    if (i >= kStages && !wait_i(bar_empty + 8 * s, uint32_t(i / kStages - 1) & 1u, abort_flag))
      return false;
    if (kb == 0) {
      const int b = ti & 1;
      if (ti >= 2 && !wait_i(bar_sempty + 8 * b, uint32_t(ti / 2 - 1) & 1u, abort_flag))
        return false;
      const int rows = n_rows - tile * kTileRows < kTileRows ? n_rows - tile * kTileRows
                                                            : kTileRows;
      const uint32_t bytes = uint32_t(rows * groups * 2);
      mbar_arrive_expect_tx(bar_sfull + 8 * b, bytes);
      bulk_load(smem_u32(stiles + b * stile_bytes), scales + size_t(tile) * kTileRows * groups,
                bytes, bar_sfull + 8 * b);
    }
    mbar_arrive_expect_tx(bar_full + 8 * s, kStageBytes);
    tma_load_2d(smem_u32(ring + s * kStageBytes), &tmap_w, kb * kKB, tile * kTileRows,
                bar_full + 8 * s);
    return true;
  };
  if (warp == 0 && lane == 0) {
    for (int i = 0; i < first; ++i) issue(i);
  }

  // ---- x as integer limbs (all threads), after the producing kernel.
  pdl_wait_primary();
  for (int i = threadIdx.x; i < num_kb * kLimbBlock / 16; i += kThreads) {
    reinterpret_cast<uint4*>(limbs)[i] = make_uint4(0, 0, 0, 0);
  }
  __syncthreads();
  const uint16_t* xb = reinterpret_cast<const uint16_t*>(input);
  for (int g = warp; g < groups; g += kThreads / 32) {
    const uint32_t v0 = xb[g * 64 + lane], v1 = xb[g * 64 + 32 + lane];
    const int e0 = int((v0 >> 7) & 0xFF), e1 = int((v1 >> 7) & 0xFF);
    int emax = e0 > e1 ? e0 : e1;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const int o = __shfl_xor_sync(0xffffffffu, emax, off);
      emax = o > emax ? o : emax;
    }
    if (lane == 0) {
      // 2^(E - 147) as a float (0 for an all-zero / subnormal group).
      const int be = emax - 147 + 127;
      gfac[g] = (emax == 0 || be <= 0) ? 0.0f : __int_as_float(be << 23);
    }
    const uint32_t vs[2] = {v0, v1};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t v = vs[h];
      const int e = int((v >> 7) & 0xFF);
      int a = 0;
      if (e != 0 && emax != 0) {
        const int mant = int(v & 0x7F) | 0x80;
        const int shift = 13 - (emax - e);
        a = shift >= 0 ? (mant << shift) : (shift > -8 ? (mant >> -shift) : 0);
      }
      const int sgn = (v & 0x8000u) ? -1 : 1;
      const int kk = g * 64 + h * 32 + lane;
      unsigned char* blk = limbs + (kk / kKB) * kLimbBlock;
      const int c = kk % kKB;
      blk[sw128(0, c)] = static_cast<unsigned char>(int8_t(sgn * (a & 127)));
      blk[sw128(1, c)] = static_cast<unsigned char>(int8_t(sgn * ((a >> 7) & 127)));
      blk[sw128(2, c)] = static_cast<unsigned char>(int8_t(sgn * (a >> 14)));
    }
  }
  fence_proxy_async_smem();  // limb tile -> tensor-core reads
  __syncthreads();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      for (int i = first; i < total_steps; ++i) {
        if (!issue(i)) break;
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_i8(128, kLimbRows);
      constexpr int kStagesPerChunk = kChunkGroups * 64 / kKB;
      int cc = 0;  // chunks started so far
      for (int i = 0; i < total_steps; ++i) {
        const int s = i % kStages;
        const int kb = i % num_kb;
        const int cb = cc % kChunks;
        if (kb % kStagesPerChunk == 0) {
          // a new chunk: its TMEM buffer must have been read out
          if (!wait_i(bar_dempty + 8 * cb, (uint32_t(cc / kChunks) & 1u) ^ 1u, abort_flag)) break;
        }
        if (!wait_i(bar_full + 8 * s, uint32_t(i / kStages) & 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t a_addr = smem_u32(ring + s * kStageBytes);
        const uint32_t b_addr = smem_u32(limbs + kb * kLimbBlock);
#pragma unroll
        for (int j = 0; j < kKB / 64; ++j) {
          const int g = kb * 2 + j;
          if (g >= groups) break;
          const uint32_t d_addr =
              tmem_base + uint32_t(cb * kChunkCols + (g % kChunkGroups) * 16);
#pragma unroll
          for (int kk = 0; kk < 2; ++kk) {
            mma_i8(d_addr, desc_sw128(a_addr + j * 64 + kk * 32),
                   desc_sw128(b_addr + j * 64 + kk * 32), idesc, kk > 0 ? 1u : 0u);
          }
        }
        mma_commit(bar_empty + 8 * s);
        if (kb % kStagesPerChunk == kStagesPerChunk - 1 || kb == num_kb - 1) {
          mma_commit(bar_dfull + 8 * cb);
          ++cc;
        }
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    float best = -FLT_MAX;
    int best_index = INT_MAX;
    int cc = 0, ti = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++ti) {
      const int row = tile * kTileRows + q * 32 + lane;
      const bool valid = row < n_rows;
      const int sb = ti & 1;
      if (!__all_sync(0xffffffffu,
                      wait_i(bar_sfull + 8 * sb, uint32_t(ti / 2) & 1u, abort_flag))) {
        break;
      }
      const uint16_t* srow = reinterpret_cast<const uint16_t*>(stiles + sb * stile_bytes) +
                             (q * 32 + lane) * groups;
      float acc = 0.0f;
      bool ok = true;
      for (int g0 = 0; g0 < groups; g0 += kChunkGroups, ++cc) {
        const int ng = groups - g0 < kChunkGroups ? groups - g0 : kChunkGroups;
        float sv[kChunkGroups];
#pragma unroll
        for (int j = 0; j < kChunkGroups; ++j) {
          sv[j] = (valid && j < ng) ? __uint_as_float(uint32_t(srow[g0 + j]) << 16) : 0.0f;
        }
        const int cb = cc % kChunks;
        const bool got = __all_sync(
            0xffffffffu, wait_i(bar_dfull + 8 * cb, uint32_t(cc / kChunks) & 1u, abort_flag));
        if (!got) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t r[kChunkGroups][4];
        const uint32_t t0 = tmem_base + (uint32_t(q * 32) << 16) + uint32_t(cb * kChunkCols);
#pragma unroll
        for (int j = 0; j < kChunkGroups; ++j) {
          asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                       : "=r"(r[j][0]), "=r"(r[j][1]), "=r"(r[j][2]), "=r"(r[j][3])
                       : "r"(t0 + uint32_t(j * 16)));
        }
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_dempty + 8 * cb);
#pragma unroll
        for (int j = 0; j < kChunkGroups; ++j) {
          if (j < ng) {
            const float comb = float(int(r[j][0])) + float(int(r[j][1])) * 128.0f +
                               float(int(r[j][2])) * 16384.0f;
            acc = fmaf(comb * gfac[g0 + j], sv[j], acc);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_sempty + 8 * sb);  // scales of this tile read
      if (!ok) break;
      if (valid) {
        const float b = bias ? __bfloat162float(bias[row]) : 0.0f;
        const bf16 y = __float2bfloat16_rn(acc + b);
        output[row] = y;
        argmax_update(best, best_index, __bfloat162float(y), row);
      }
    }
    if (block_value != nullptr) {
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, off);
        const int oi = __shfl_xor_sync(0xffffffffu, best_index, off);
        argmax_update(best, best_index, ov, oi);
      }
      if (lane == 0) {
        red_v[q] = best;
        red_i[q] = best_index;
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (q == 0 && lane == 0) {
        float bv = -FLT_MAX;
        int bi = INT_MAX;
        for (int w = 0; w < 4; ++w) argmax_update(bv, bi, red_v[w], red_i[w]);
        block_value[blockIdx.x] = bv;
        block_index[blockIdx.x] = bi;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(kChunks * kChunkCols)
                 : "memory");
  }
}

int fixed_smem_bytes(int k) {
  const int num_kb = (k + kKB - 1) / kKB;
  return 1024 + num_kb * kLimbBlock + 2 * kTileRows * (k / 64) * 2 + (k / 64) * 4 + 16 +
         8 * (2 * kMaxStages + 2 * kChunks + 4) + 64;
}
constexpr int kSmemLimit = 227 * 1024;
int stages_for(int k) {
  const int st = (kSmemLimit - fixed_smem_bytes(k)) / kStageBytes;
  return st > kMaxStages ? kMaxStages : st;
}
int smem_bytes(int k) { return fixed_smem_bytes(k) + stages_for(k) * kStageBytes; }

}  // namespace

bool gemv_i8tc_supported(const void* weight, const void* input, const void* scales, int n,
                         int k) {
  // Each 128-row tile walks its K serially: the kernel pays off only when
  // there are enough tiles for every SM several times over.
  // Tile scale copies: 16-byte aligned, sizes a multiple of 16 (n % 8).
  return stages_for(k) >= 4 && n >= kMinRows && n % 8 == 0 && k >= 64 && k % 64 == 0 && k <= kMaxK &&
         (reinterpret_cast<uintptr_t>(weight) & 15u) == 0 &&
         (reinterpret_cast<uintptr_t>(input) & 15u) == 0 && scales != nullptr &&
         (reinterpret_cast<uintptr_t>(scales) & 15u) == 0;
}

int gemv_i8tc_grid(int n) {
  static std::atomic<int> sms{0};
  int c = sms.load(std::memory_order_relaxed);
  if (c == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    c = 148;
    cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev);
    sms.store(c, std::memory_order_relaxed);
  }
  const int tiles = (n + kTileRows - 1) / kTileRows;
  return tiles < c ? tiles : c;
}

cudaError_t launch_gemv_i8tc(const void* weight, const bf16* scales, const bf16* bias,
                             const bf16* input, bf16* output, int n, int k, float* block_value,
                             int* block_index, cudaStream_t stream, int* grid_out) {
  CUtensorMap tw;
  if (!encode_tmap_2d(&tw, weight, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, k, n, kKB, kTileRows,
                      CU_TENSOR_MAP_SWIZZLE_128B)) {
    return cudaErrorInvalidValue;
  }
  const int smem = smem_bytes(k);
  static std::atomic<unsigned long long> attr_done{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = (dev >= 0 && dev < 64) ? 1ull << dev : 0ull;
  if (bit == 0 || (attr_done.load(std::memory_order_acquire) & bit) == 0) {
    const cudaError_t e = cudaFuncSetAttribute(
        gemv_i8tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
    if (e != cudaSuccess) return e;
    attr_done.fetch_or(bit, std::memory_order_release);
  }
  const int grid = gemv_i8tc_grid(n);
  if (grid_out) *grid_out = grid;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemv_i8tc_kernel, tw,
                            reinterpret_cast<const uint16_t*>(scales), bias, input, output, n, k,
                            block_value, block_index, stages_for(k));
}

}  // namespace b200
