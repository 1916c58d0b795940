// W8A16 prefill GEMM with the dequantised weights held in TENSOR MEMORY.
//
//   Y[M,N] = bf16( X[M,K] . bf16(q[N,K] * s[N,K/64])^T + b[N] )
//
// computed as its transpose, Y^T = W . X^T, so that the weight tile is the
// MMA's A operand and can live in TMEM instead of shared memory:
//   * TMA brings raw INT8 weight tiles [128 rows x 64] (64-byte swizzle) and
//     X tiles [kBT tokens x 64] BF16 (128-byte swizzle) into a shared-memory
//     ring;
//   * eight dequantiser warps turn each INT8 tile into bf16(q*s) in
//     registers and write it with tcgen05.st into a ring of A slots in TMEM
//     (row r of the tile = TMEM lane r; 64 K values = 32 columns of BF16
//     pairs).  The dequantised weights never touch shared memory: per k-block
//     the SMEM traffic is the X tile (TMA write + MMA read) plus the 8 KB INT8
//     tile, instead of also writing and reading a 16 KB BF16 weight tile;
//   * one thread issues tcgen05.mma.cta_group::1.kind::f16 with A from TMEM
//     and B (= the X tile, K-major) from shared memory: D[128 x kBT] FP32 in
//     TMEM, double-buffered across tiles;
//   * four epilogue warps read D with tcgen05.ld (lane = output feature n,
//     column = token), add the bias (one value per thread), round to BF16
//     and store Y rows (pairs of features exchanged between neighbouring
//     lanes so every store is 4 bytes and a warp writes two 64-byte row
//     segments).
//
// The BF16 rounding of q*s and the K order (16 at a time, k ascending) are
// those of the reference's tensor-core GEMM (src/cuda/kernels.cu:1075-1094,
// 1096-1322), so results equal the other GEMM paths of this library.
//
// TMEM: 512 columns = 2 accumulators of kBT columns + kAStages A slots of 32.
// Warps: 0 TMA producer, 1 TMEM allocator + MMA issuer, 4..7 epilogue,
// 8..15 dequantisers (warp w reaches TMEM lanes 32*(w%4)..+31; warps w and
// w+4 split the 64 K values of a k-block).  Every wait is bounded and
// reports B200_DEVICE_TIMEOUT_* like the other GEMM kernels.  No multicast.

#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace b200 {

__device__ int g_w8t_status = 0;

cudaError_t read_w8t_status(int* value, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(value, g_w8t_status, sizeof(int));
  if (e != cudaSuccess || !clear) return e;
  const int zero = 0;
  return cudaMemcpyToSymbol(g_w8t_status, &zero, sizeof(int));
}

// Tensor-map encoder with the per-call cache (gemm_sm100.cu).
bool encode_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                    int elem_bytes, int inner, int outer, int box_inner, int box_outer,
                    CUtensorMapSwizzle swizzle);

namespace {

constexpr int kRows = 128;   // weight rows (output features) per tile
constexpr int kBK = 64;      // K per k-block = one quantisation group
// kSub: quantisation groups (64 K values) per pipeline stage, 1 or 2.  The
// MMA issuer pays a fixed ~300-500 cycles per barrier wait (measured), so a
// stage must carry enough MMA work to keep the tensor pipe busy meanwhile.
// kW16: BF16 weights, loaded by TMA as [128 x 64] 128-byte-swizzled
// sub-tiles and read by the MMA from shared memory (no dequantiser warps,
// no A slots in TMEM); the rest of the kernel is shared.
template <int kBT, int kSub, bool kW16 = false>
struct CfgT {
  static constexpr int kKS = kBK * kSub;                  // K per stage
  static constexpr int kDqWarps = kW16 ? 0 : 8;           // 2 per lane quarter
  static constexpr int kXSub = kBT * kBK * 2;             // one 64-wide X sub-tile
  static constexpr int kXBytes = kSub * kXSub;
  static constexpr int kWSub = kRows * kBK * 2;           // one BF16 W sub-tile
  static constexpr int kQBytes = kW16 ? kSub * kWSub : kRows * kKS;  // W tile
  static constexpr int kStageBytes = kXBytes + kQBytes;
  static constexpr int kStages =
      (200 * 1024) / kStageBytes > 8 ? 8 : (200 * 1024) / kStageBytes;
  static constexpr int kAccCols = kBT;
  static constexpr int kACols = kKS / 2;                  // BF16 pairs per slot
  static constexpr int kAStages =
      kW16 ? 1 : ((512 - 2 * kAccCols) / kACols > 8 ? 8 : (512 - 2 * kAccCols) / kACols);
  static constexpr int kACol0 = 2 * kAccCols;
  static constexpr int kThreads = (8 + kDqWarps) * 32;
  static constexpr int kSmemBytes = kStages * kStageBytes + 512 + 1024;
  static_assert(kSub == 1 || kSub == 2, "one or two groups per stage");
  static_assert(kBT % 16 == 0 && kBT >= 16 && kBT <= 256, "MMA N");
  static_assert((kW16 || kAStages >= 2) && kStages >= 2, "ring sizes");
  static_assert(kXSub % 1024 == 0, "128B-swizzle atoms");
};

__device__ __forceinline__ bool wait_t(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                       int code) {
  return mbar_wait_bounded(bar, parity, abort_flag, code, &g_w8t_status);
}

// bf16(q * s) of the four int8 of `word` -> two packed BF16 pairs.
__device__ __forceinline__ void dq4(uint32_t word, bf162 s2, uint32_t* out) {
  const uint32_t b = word ^ 0x80808080u;
  const float2 q01 = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(b, 0x4B000000u, 0x7540u)),
                                            __uint_as_float(__byte_perm(b, 0x4B000000u, 0x7541u))),
                                make_float2(-8388736.0f, -8388736.0f));
  const float2 q23 = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(b, 0x4B000000u, 0x7542u)),
                                            __uint_as_float(__byte_perm(b, 0x4B000000u, 0x7543u))),
                                make_float2(-8388736.0f, -8388736.0f));
  // q has <= 8 significant bits: its BF16 is the top half of the float.
  uint32_t p01 = __byte_perm(__float_as_uint(q01.x), __float_as_uint(q01.y), 0x7632);
  uint32_t p23 = __byte_perm(__float_as_uint(q23.x), __float_as_uint(q23.y), 0x7632);
  const bf162 neg0 = __halves2bfloat162(__ushort_as_bfloat16(0x8000), __ushort_as_bfloat16(0x8000));
  // q*s is exact in FP32; fma.rn.bf16x2(q, s, -0) rounds it to BF16 once.
  const bf162 d01 = __hfma2(*reinterpret_cast<bf162*>(&p01), s2, neg0);
  const bf162 d23 = __hfma2(*reinterpret_cast<bf162*>(&p23), s2, neg0);
  out[0] = *reinterpret_cast<const uint32_t*>(&d01);
  out[1] = *reinterpret_cast<const uint32_t*>(&d23);
}

template <int kBT, int kSub, bool kW16>
__global__ void __launch_bounds__(CfgT<kBT, kSub, kW16>::kThreads, 1)
gemm_w8t_kernel(const __grid_constant__ CUtensorMap tmap_x,
                const __grid_constant__ CUtensorMap tmap_q,
                const uint16_t* __restrict__ scales, const bf16* __restrict__ bias,
                bf16* __restrict__ out, int m, int n, int k, int ldc,
                const unsigned char* __restrict__ packed) {
  using C = CfgT<kBT, kSub, kW16>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
  // full[S], empty[S], a_full[A], a_empty[A], acc_full[2], acc_empty[2]
  const uint32_t bar_full = smem_u32(bars);
  const uint32_t bar_empty = bar_full + 8 * C::kStages;
  const uint32_t bar_afull = bar_empty + 8 * C::kStages;
  const uint32_t bar_aempty = bar_afull + 8 * C::kAStages;
  const uint32_t bar_acc_full = bar_aempty + 8 * C::kAStages;
  const uint32_t bar_acc_empty = bar_acc_full + 16;
  uint32_t* tmem_slot =
      reinterpret_cast<uint32_t*>(bars + 2 * C::kStages + 2 * C::kAStages + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (m + kBT - 1) / kBT;
  const int num_n = (n + kRows - 1) / kRows;
  const int num_tiles = num_m * num_n;
  const int num_kb = (k + C::kKS - 1) / C::kKS;
  const int groups = (k + 63) / 64;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1 + C::kDqWarps);  // MMA commit + dequant warps
    }
    for (int a = 0; a < C::kAStages; ++a) {
      mbar_init(bar_afull + 8 * a, C::kDqWarps > 0 ? C::kDqWarps : 1);  // unused: kW16
      mbar_init(bar_aempty + 8 * a, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar_acc_full + 8 * b, 1);
      mbar_init(bar_acc_empty + 8 * b, 128);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Programmatic dependent launch: the set-up above overlaps the previous
  // kernel; X (and the output) are touched only after it has completed.
  pdl_launch_dependents();
  pdl_wait_primary();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
        const int mb = tile % num_m;
        const int nb = tile / num_m;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!wait_t(bar_empty + 8 * stage, phase ^ 1, abort_flag,
                      B200_DEVICE_TIMEOUT_PIPELINE))
            goto producer_done;
          unsigned char* st = smem + stage * C::kStageBytes;
          const uint32_t fb = bar_full + 8 * stage;
          mbar_arrive_expect_tx(fb, C::kStageBytes);
#pragma unroll
          for (int sub = 0; sub < kSub; ++sub) {
            tma_load_2d(smem_u32(st + sub * C::kXSub), &tmap_x, kb * C::kKS + sub * kBK,
                        mb * kBT, fb);
          }
          if constexpr (kW16) {
#pragma unroll
            for (int sub = 0; sub < kSub; ++sub) {
              tma_load_2d(smem_u32(st + C::kXBytes + sub * C::kWSub), &tmap_q,
                          kb * C::kKS + sub * kBK, nb * kRows, fb);
            }
          } else if (kSub == 2 && packed != nullptr) {
            // Pre-packed weights: the tile's shared-memory image is one
            // contiguous 16 KB block (b200_pack_w8a16).
            bulk_load(smem_u32(st + C::kXBytes),
                      packed + (size_t(nb) * num_kb + kb) * C::kQBytes, C::kQBytes, fb);
          } else {
            tma_load_2d(smem_u32(st + C::kXBytes), &tmap_q, kb * C::kKS, nb * kRows, fb);
          }
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  producer_done:;
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(128, kBT);
      int stage = 0, aslot = 0;
      uint32_t phase = 0, aphase = 0;
      int it = 0;
      for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++it) {
        const int buf = it & 1;
        const uint32_t use = (it >> 1) & 1;
        if (!wait_t(bar_acc_empty + 8 * buf, use ^ 1, abort_flag, B200_DEVICE_TIMEOUT_ACCUM))
          break;
        tc_fence_after();
        const uint32_t d_addr = tmem_base + uint32_t(buf * C::kAccCols);
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          // The dequant warps arrive on a_full only after they waited for
          // this step's stage (X and INT8 land on the same barrier), so a_full
          // also orders the X tile: one wait per k-block.
          // kW16: the stage's own full barrier (X and W land on it).
          if (!wait_t(kW16 ? bar_full + 8 * stage : bar_afull + 8 * aslot,
                      kW16 ? phase : aphase, abort_flag, B200_DEVICE_TIMEOUT_PIPELINE)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t x_addr = smem_u32(smem + stage * C::kStageBytes);
          if constexpr (kW16) {
            const uint32_t w_addr = x_addr + C::kXBytes;
#pragma unroll
            for (int kk = 0; kk < C::kKS / 16; ++kk) {
              mma_bf16(d_addr, desc_sw128(w_addr + (kk >> 2) * C::kWSub + (kk & 3) * 32),
                       desc_sw128(x_addr + (kk >> 2) * C::kXSub + (kk & 3) * 32), idesc,
                       (kb > 0 || kk > 0) ? 1u : 0u);
            }
            mma_commit(bar_empty + 8 * stage);
          } else {
            const uint32_t a_addr = tmem_base + uint32_t(C::kACol0 + aslot * C::kACols);
#pragma unroll
            for (int kk = 0; kk < C::kKS / 16; ++kk) {
              mma_bf16_ta(d_addr, a_addr + uint32_t(kk * 8),
                          desc_sw128(x_addr + (kk >> 2) * C::kXSub + (kk & 3) * 32), idesc,
                          (kb > 0 || kk > 0) ? 1u : 0u);
            }
            mma_commit(bar_empty + 8 * stage);
            mma_commit(bar_aempty + 8 * aslot);
          }
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
          if (++aslot == C::kAStages) {
            aslot = 0;
            aphase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit(bar_acc_full + 8 * buf);
      }
    }
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const bool pairs_ok = (ldc % 2 == 0) && (n % 2 == 0) &&
                          ((reinterpret_cast<uintptr_t>(out) & 3u) == 0);
    int it = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++it) {
      const int mb = tile % num_m;
      const int nb = tile / num_m;
      const int buf = it & 1;
      const uint32_t use = (it >> 1) & 1;
      const bool acc_ok =
          wait_t(bar_acc_full + 8 * buf, use, abort_flag, B200_DEVICE_TIMEOUT_ACCUM);
      if (!__all_sync(0xffffffffu, acc_ok)) break;
      tc_fence_after();
      const int feat = nb * kRows + q * 32 + lane;  // this thread's output feature
      const float bv = (bias != nullptr && feat < n) ? __bfloat162float(bias[feat]) : 0.0f;
      const bool odd = (lane & 1) != 0;
      const bool feat_pair_ok = feat - (odd ? 1 : 0) < n;
      // 16 columns (tokens) per tcgen05.ld: few live registers.
#pragma unroll 1
      for (int c0 = 0; c0 < kBT; c0 += 16) {
        uint32_t r[16];
        tmem_ld16(tmem_base + (uint32_t(q * 32) << 16) + uint32_t(buf * C::kAccCols + c0), r);
        const int tok0 = mb * kBT + c0;
        if (pairs_ok) {
          bf16* rowp = out + size_t(tok0 + (odd ? 1 : 0)) * ldc + (feat - (odd ? 1 : 0));
#pragma unroll
          for (int j = 0; j < 16; j += 2) {
            const float v0 = __uint_as_float(r[j]) + bv;      // token tok0 + j
            const float v1 = __uint_as_float(r[j + 1]) + bv;  // token tok0 + j + 1
            // even lane keeps token j and takes its odd neighbour's token j;
            // odd lane keeps token j+1 and takes its even neighbour's j+1.
            const float got = __shfl_xor_sync(0xffffffffu, odd ? v0 : v1, 1);
            const bf162 h = odd ? __floats2bfloat162_rn(got, v1) : __floats2bfloat162_rn(v0, got);
            const int tok = tok0 + j + (odd ? 1 : 0);
            if (tok < m && feat_pair_ok) {
              *reinterpret_cast<bf162*>(rowp + size_t(j) * ldc) = h;
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int tok = tok0 + j;
            if (tok < m && feat < n) {
              out[size_t(tok) * ldc + feat] = __float2bfloat16_rn(__uint_as_float(r[j]) + bv);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(bar_acc_empty + 8 * buf);
    }
  } else if (!kW16 && warp >= 8) {
    // ---------------------------------------------------------- dequantiser
    // Warps w and w+4 cover TMEM lane quarter w % 4 and split each stage's K
    // range in two parts (part p: kKS/2 values = one group when kSub == 2).
    const int dw = warp - 8;
    const int quarter = dw & 3;
    const int part = dw >> 2;
    const int rl = quarter * 32 + lane;  // row of the tile = TMEM lane
    const uint32_t t_lane = uint32_t(quarter * 32) << 16;
    // INT8 tile swizzle: 64-byte rows (kSub 1): chunk c at c ^ ((r >> 1) & 3);
    // 128-byte rows (kSub 2): chunk c at c ^ (r & 7).
    const int sw = kSub == 1 ? ((rl >> 1) & 3) : (rl & 7);
    constexpr int kChunks = kSub * 2;  // 16-byte chunks per thread per stage
    int stage = 0, aslot = 0;
    uint32_t phase = 0, aphase = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
      const int row = (tile / num_m) * kRows + rl;
      const bool srow_ok = row < n;
      const uint16_t* srow = scales + size_t(srow_ok ? row : 0) * groups;
      // group of this thread's part in k-block kb: kb * kSub + part (kSub 2)
      // or kb (kSub 1)
      auto group_of = [&](int kb) { return kSub == 2 ? kb * 2 + part : kb; };
      uint32_t s_next = (srow_ok && group_of(0) < groups) ? srow[group_of(0)] : 0u;
      for (int kb = 0; kb < num_kb; ++kb) {
        const uint32_t sv = s_next;
        if (kb + 1 < num_kb) {
          const int g1 = group_of(kb + 1);
          s_next = (srow_ok && g1 < groups) ? srow[g1] : 0u;
        }
        if (!wait_t(bar_full + 8 * stage, phase, abort_flag, B200_DEVICE_TIMEOUT_PIPELINE)) {
          ok = false;
          break;
        }
        const unsigned char* qt = smem + stage * C::kStageBytes + C::kXBytes + rl * C::kKS;
        uint4 c[kChunks];
#pragma unroll
        for (int j = 0; j < kChunks; ++j) {
          c[j] = *reinterpret_cast<const uint4*>(qt + (((part * kChunks + j) ^ sw) << 4));
        }
        const uint32_t s2bits = sv | (sv << 16);
        const bf162 s2 = *reinterpret_cast<const bf162*>(&s2bits);
        uint32_t v[8 * kChunks];
#pragma unroll
        for (int j = 0; j < kChunks; ++j) {
          dq4(c[j].x, s2, v + 8 * j + 0);
          dq4(c[j].y, s2, v + 8 * j + 2);
          dq4(c[j].z, s2, v + 8 * j + 4);
          dq4(c[j].w, s2, v + 8 * j + 6);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_empty + 8 * stage);  // INT8 tile consumed
        if (!wait_t(bar_aempty + 8 * aslot, aphase ^ 1, abort_flag,
                    B200_DEVICE_TIMEOUT_PIPELINE)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t ta = tmem_base + t_lane +
                            uint32_t(C::kACol0 + aslot * C::kACols + part * (C::kACols / 2));
#pragma unroll
        for (int j = 0; j < kChunks / 2; ++j) tmem_st16(ta + 16 * j, v + 16 * j);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_afull + 8 * aslot);
        if (++stage == C::kStages) {
          stage = 0;
          phase ^= 1;
        }
        if (++aslot == C::kAStages) {
          aslot = 0;
          aphase ^= 1;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(512)
                 : "memory");
  }
}

template <int kBT, int kSub, bool kW16 = false>
cudaError_t launch_bt(const void* weight, const bf16* scales, const bf16* bias,
                      const bf16* input, bf16* output, int m, int n, int k, int ldc,
                      cudaStream_t stream, const void* packed = nullptr) {
  using C = CfgT<kBT, kSub, kW16>;
  CUtensorMap tx, tq;
  if (!encode_tmap_2d(&tx, input, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, k, m, kBK, kBT,
                      CU_TENSOR_MAP_SWIZZLE_128B) ||
      !(kW16 ? encode_tmap_2d(&tq, weight, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, k, n, kBK,
                              kRows, CU_TENSOR_MAP_SWIZZLE_128B)
             : encode_tmap_2d(&tq, weight, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, k, n, C::kKS,
                              kRows,
                              kSub == 1 ? CU_TENSOR_MAP_SWIZZLE_64B
                                        : CU_TENSOR_MAP_SWIZZLE_128B))) {
    return cudaErrorInvalidValue;
  }
  static std::atomic<unsigned long long> attr_done{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = (dev >= 0 && dev < 64) ? 1ull << dev : 0ull;
  if (bit == 0 || (attr_done.load(std::memory_order_acquire) & bit) == 0) {
    const cudaError_t e = cudaFuncSetAttribute(
        gemm_w8t_kernel<kBT, kSub, kW16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
        C::kSmemBytes);
    if (e != cudaSuccess) return e;
    attr_done.fetch_or(bit, std::memory_order_release);
  }
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int tiles = ((m + kBT - 1) / kBT) * ((n + kRows - 1) / kRows);
  const int grid = tiles < sms ? tiles : sms;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(C::kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemm_w8t_kernel<kBT, kSub, kW16>, tx, tq,
                            reinterpret_cast<const uint16_t*>(scales), bias, output, m, n, k,
                            ldc, static_cast<const unsigned char*>(packed));
}

// ===================================================================
// CTA-pair form (cta_group::2): one tile = 256 weight rows x kBT tokens per
// pair of SMs.  Each CTA dequantises its own 128 weight rows into its own
// TMEM A slots (as above) and loads HALF of the X tile (kBT/2 tokens); the
// leader CTA issues tcgen05.mma.cta_group::2 (M = 256, N = kBT) with A from
// each CTA's TMEM and B from both X halves, D = each CTA's 128 rows x kBT.
// Per SM this halves the X traffic through shared memory (TMA write + MMA
// read), which bounds the one-SM form: its BF16 twin, with no dequantiser
// at all, reaches only 700-980 TF/s.
//
// Barriers (same offsets in both CTAs):
//   full[s]    each CTA: its INT8 tile; the leader's also receives both X
//              halves (the .cta_group::2 TMA form routes the peer's bytes
//              to the leader), so the leader's dequantisers also order X;
//   empty[s]   each CTA: the leader's commit (multicast) + its 8
//              dequantiser warps;
//   a_full[a]  leader: 16 arrivals, 8 local warps + 8 remote (relaxed,
//              after tcgen05.wait::st and fence::before_thread_sync);
//   a_empty[a] each CTA: commit multicast;
//   acc_full   each CTA: commit multicast; acc_empty leader, one arrival
//              per CTA after its four epilogue warps meet.
// No TMA multicast.  Every wait is bounded (2 s) and reports
// B200_DEVICE_TIMEOUT_*.
// ===================================================================
template <int kBT>
struct CfgP {
  static constexpr int kSub = 2;
  static constexpr int kKS = kBK * kSub;                  // K per stage
  static constexpr int kDqWarps = 8;
  static constexpr int kXHalf = kBT / 2;                  // tokens per CTA
  static constexpr int kXSub = kXHalf * kBK * 2;          // one 64-wide X half sub-tile
  static constexpr int kXBytes = kSub * kXSub;
  static constexpr int kQBytes = kRows * kKS;
  static constexpr int kStageBytes = kXBytes + kQBytes;
  static constexpr int kStages =
      (200 * 1024) / kStageBytes > 8 ? 8 : (200 * 1024) / kStageBytes;
  static constexpr int kAccCols = kBT;
  static constexpr int kACols = kKS / 2;
  static constexpr int kAStages =
      (512 - 2 * kAccCols) / kACols > 8 ? 8 : (512 - 2 * kAccCols) / kACols;
  static constexpr int kACol0 = 2 * kAccCols;
  static constexpr int kThreads = (8 + kDqWarps) * 32;
  static constexpr int kSmemBytes = kStages * kStageBytes + 512 + 1024;
  static_assert(kBT % 32 == 0 && kBT <= 256, "pair MMA N, 16-row halves");
  static_assert(kAStages >= 2 && kStages >= 2, "ring sizes");
  static_assert(kXSub % 1024 == 0, "128B-swizzle atoms");
};

__device__ __forceinline__ bool wait_tc(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                        int code) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  while (true) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if (*abort_flag) return false;
    if (global_timer_ns() - start > kWaitTimeoutNs) {
      *abort_flag = 1;
      atomicCAS(&g_w8t_status, 0, code);
      return false;
    }
  }
}

template <int kBT>
__global__ void __launch_bounds__(CfgP<kBT>::kThreads, 1)
gemm_w8t2_kernel(const __grid_constant__ CUtensorMap tmap_x,
                 const __grid_constant__ CUtensorMap tmap_q,
                 const uint16_t* __restrict__ scales, const bf16* __restrict__ bias,
                 bf16* __restrict__ out, int m, int n, int k, int ldc,
                 const unsigned char* __restrict__ packed) {
  using C = CfgP<kBT>;
  extern __shared__ __align__(1024) unsigned char smem_rawp[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_rawp) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
  const uint32_t bar_full = smem_u32(bars);
  const uint32_t bar_empty = bar_full + 8 * C::kStages;
  const uint32_t bar_afull = bar_empty + 8 * C::kStages;
  const uint32_t bar_aempty = bar_afull + 8 * C::kAStages;
  const uint32_t bar_acc_full = bar_aempty + 8 * C::kAStages;
  const uint32_t bar_acc_empty = bar_acc_full + 16;
  uint32_t* tmem_slot =
      reinterpret_cast<uint32_t*>(bars + 2 * C::kStages + 2 * C::kAStages + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster = blockIdx.x >> 1;
  const int num_clusters = gridDim.x >> 1;
  const int num_m = (m + kBT - 1) / kBT;
  const int num_n = (n + 2 * kRows - 1) / (2 * kRows);
  const int num_tiles = num_m * num_n;
  const int num_kb = (k + C::kKS - 1) / C::kKS;
  const int groups = (k + 63) / 64;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1 + C::kDqWarps);
    }
    for (int a = 0; a < C::kAStages; ++a) {
      mbar_init(bar_afull + 8 * a, 2 * C::kDqWarps);
      mbar_init(bar_aempty + 8 * a, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar_acc_full + 8 * b, 1);
      mbar_init(bar_acc_empty + 8 * b, 2);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile(
        "tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
            smem_u32(tmem_slot)),
        "r"(512)
        : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_launch_dependents();
  pdl_wait_primary();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = cluster; tile < num_tiles; tile += num_clusters) {
        const int mb = tile % num_m;
        const int nb = tile / num_m;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!wait_tc(bar_empty + 8 * stage, phase ^ 1, abort_flag,
                       B200_DEVICE_TIMEOUT_PIPELINE))
            goto producer_done;
          unsigned char* st = smem + stage * C::kStageBytes;
          const uint32_t fb = bar_full + 8 * stage;
          mbar_arrive_expect_tx(fb, leader ? 2 * C::kXBytes + C::kQBytes : C::kQBytes);
#pragma unroll
          for (int sub = 0; sub < C::kSub; ++sub) {
            tma_load_2d_pair(smem_u32(st + sub * C::kXSub), &tmap_x, kb * C::kKS + sub * kBK,
                             mb * kBT + int(rank) * C::kXHalf, fb);
          }
          if (packed != nullptr) {
            bulk_load(smem_u32(st + C::kXBytes),
                      packed + (size_t(nb * 2 + int(rank)) * num_kb + kb) * C::kQBytes,
                      C::kQBytes, fb);
          } else {
            tma_load_2d(smem_u32(st + C::kXBytes), &tmap_q, kb * C::kKS,
                        nb * 2 * kRows + int(rank) * kRows, fb);
          }
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  producer_done:;
  } else if (warp == 1) {
    // ------------------------------------------------------ MMA (leader)
    if (leader && lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(256, kBT);
      int stage = 0, aslot = 0;
      uint32_t aphase = 0;
      int it = 0;
      for (int tile = cluster; tile < num_tiles; tile += num_clusters, ++it) {
        const int buf = it & 1;
        const uint32_t use = (it >> 1) & 1;
        if (!wait_tc(bar_acc_empty + 8 * buf, use ^ 1, abort_flag, B200_DEVICE_TIMEOUT_ACCUM))
          break;
        tc_fence_after();
        const uint32_t d_addr = tmem_base + uint32_t(buf * C::kAccCols);
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          // a_full: both CTAs' A slots written; the leader's dequantisers
          // arrive only after its full[s] (which carries both X halves).
          if (!wait_tc(bar_afull + 8 * aslot, aphase, abort_flag,
                       B200_DEVICE_TIMEOUT_PIPELINE)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t x_addr = smem_u32(smem + stage * C::kStageBytes);
          const uint32_t a_addr = tmem_base + uint32_t(C::kACol0 + aslot * C::kACols);
#pragma unroll
          for (int kk = 0; kk < C::kKS / 16; ++kk) {
            mma2_bf16_ta(d_addr, a_addr + uint32_t(kk * 8),
                         desc_sw128(x_addr + (kk >> 2) * C::kXSub + (kk & 3) * 32), idesc,
                         (kb > 0 || kk > 0) ? 1u : 0u);
          }
          mma2_commit_both(bar_empty + 8 * stage);
          mma2_commit_both(bar_aempty + 8 * aslot);
          if (++stage == C::kStages) stage = 0;
          if (++aslot == C::kAStages) {
            aslot = 0;
            aphase ^= 1;
          }
        }
        if (!ok) break;
        mma2_commit_both(bar_acc_full + 8 * buf);
      }
    }
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const bool pairs_ok = (ldc % 2 == 0) && (n % 2 == 0) &&
                          ((reinterpret_cast<uintptr_t>(out) & 3u) == 0);
    const uint32_t acc_empty_leader = map_to_rank(bar_acc_empty, 0);
    int it = 0;
    for (int tile = cluster; tile < num_tiles; tile += num_clusters, ++it) {
      const int mb = tile % num_m;
      const int nb = tile / num_m;
      const int buf = it & 1;
      const uint32_t use = (it >> 1) & 1;
      // A failed wait skips the work but keeps the four warps in step with
      // the named barrier below (warp-uniform: tcgen05.ld needs the warp).
      const bool acc_ok = __all_sync(
          0xffffffffu,
          wait_tc(bar_acc_full + 8 * buf, use, abort_flag, B200_DEVICE_TIMEOUT_ACCUM));
      tc_fence_after();
      const int feat = nb * 2 * kRows + int(rank) * kRows + q * 32 + lane;
      const float bv = (bias != nullptr && feat < n) ? __bfloat162float(bias[feat]) : 0.0f;
      const bool odd = (lane & 1) != 0;
      const bool feat_pair_ok = feat - (odd ? 1 : 0) < n;
#pragma unroll 1
      for (int c0 = 0; acc_ok && c0 < kBT; c0 += 16) {
        uint32_t r[16];
        tmem_ld16(tmem_base + (uint32_t(q * 32) << 16) + uint32_t(buf * C::kAccCols + c0), r);
        const int tok0 = mb * kBT + c0;
        if (pairs_ok) {
          bf16* rowp = out + size_t(tok0 + (odd ? 1 : 0)) * ldc + (feat - (odd ? 1 : 0));
#pragma unroll
          for (int j = 0; j < 16; j += 2) {
            const float v0 = __uint_as_float(r[j]) + bv;
            const float v1 = __uint_as_float(r[j + 1]) + bv;
            const float got = __shfl_xor_sync(0xffffffffu, odd ? v0 : v1, 1);
            const bf162 h = odd ? __floats2bfloat162_rn(got, v1) : __floats2bfloat162_rn(v0, got);
            const int tok = tok0 + j + (odd ? 1 : 0);
            if (tok < m && feat_pair_ok) {
              *reinterpret_cast<bf162*>(rowp + size_t(j) * ldc) = h;
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int tok = tok0 + j;
            if (tok < m && feat < n) {
              out[size_t(tok) * ldc + feat] = __float2bfloat16_rn(__uint_as_float(r[j]) + bv);
            }
          }
        }
      }
      tc_fence_before();
      asm volatile("bar.sync 3, 128;" ::: "memory");
      if (threadIdx.x == 4 * 32) {
        if (leader) {
          mbar_arrive(bar_acc_empty + 8 * buf);
        } else {
          mbar_arrive_remote(acc_empty_leader + 8 * buf);
        }
      }
    }
  } else if (warp >= 8) {
    // ---------------------------------------------------------- dequantiser
    // As in the one-SM form: warps w and w+4 cover TMEM lane quarter w % 4
    // and split each stage's 128 K values into one group each.
    const int dw = warp - 8;
    const int quarter = dw & 3;
    const int part = dw >> 2;
    const int rl = quarter * 32 + lane;
    const uint32_t t_lane = uint32_t(quarter * 32) << 16;
    const int sw = rl & 7;  // 128-byte swizzle of the INT8 tile
    constexpr int kChunks = 4;
    const uint32_t afull_leader = map_to_rank(bar_afull, 0);
    int stage = 0, aslot = 0;
    uint32_t phase = 0, aphase = 0;
    bool ok = true;
    for (int tile = cluster; ok && tile < num_tiles; tile += num_clusters) {
      const int row = (tile / num_m) * 2 * kRows + int(rank) * kRows + rl;
      const bool srow_ok = row < n;
      const uint16_t* srow = scales + size_t(srow_ok ? row : 0) * groups;
      auto group_of = [&](int kb) { return kb * 2 + part; };
      uint32_t s_next = (srow_ok && group_of(0) < groups) ? srow[group_of(0)] : 0u;
      for (int kb = 0; kb < num_kb; ++kb) {
        const uint32_t sv = s_next;
        if (kb + 1 < num_kb) {
          const int g1 = group_of(kb + 1);
          s_next = (srow_ok && g1 < groups) ? srow[g1] : 0u;
        }
        if (!wait_tc(bar_full + 8 * stage, phase, abort_flag, B200_DEVICE_TIMEOUT_PIPELINE)) {
          ok = false;
          break;
        }
        const unsigned char* qt = smem + stage * C::kStageBytes + C::kXBytes + rl * C::kKS;
        uint4 c[kChunks];
#pragma unroll
        for (int j = 0; j < kChunks; ++j) {
          c[j] = *reinterpret_cast<const uint4*>(qt + (((part * kChunks + j) ^ sw) << 4));
        }
        const uint32_t s2bits = sv | (sv << 16);
        const bf162 s2 = *reinterpret_cast<const bf162*>(&s2bits);
        uint32_t v[8 * kChunks];
#pragma unroll
        for (int j = 0; j < kChunks; ++j) {
          dq4(c[j].x, s2, v + 8 * j + 0);
          dq4(c[j].y, s2, v + 8 * j + 2);
          dq4(c[j].z, s2, v + 8 * j + 4);
          dq4(c[j].w, s2, v + 8 * j + 6);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_empty + 8 * stage);  // INT8 tile consumed
        if (!wait_tc(bar_aempty + 8 * aslot, aphase ^ 1, abort_flag,
                     B200_DEVICE_TIMEOUT_PIPELINE)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t ta = tmem_base + t_lane +
                            uint32_t(C::kACol0 + aslot * C::kACols + part * (C::kACols / 2));
#pragma unroll
        for (int j = 0; j < kChunks / 2; ++j) tmem_st16(ta + 16 * j, v + 16 * j);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (leader) {
            mbar_arrive(bar_afull + 8 * aslot);
          } else {
            mbar_arrive_remote_relaxed(afull_leader + 8 * aslot);
          }
        }
        if (++stage == C::kStages) {
          stage = 0;
          phase ^= 1;
        }
        if (++aslot == C::kAStages) {
          aslot = 0;
          aphase ^= 1;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(512)
                 : "memory");
  }
}

template <int kBT>
cudaError_t launch_pair_bt(const void* weight, const bf16* scales, const bf16* bias,
                           const bf16* input, bf16* output, int m, int n, int k, int ldc,
                           cudaStream_t stream, const void* packed = nullptr) {
  using C = CfgP<kBT>;
  CUtensorMap tx, tq;
  if (!encode_tmap_2d(&tx, input, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, k, m, kBK, C::kXHalf,
                      CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_tmap_2d(&tq, weight, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, k, n, C::kKS, kRows,
                      CU_TENSOR_MAP_SWIZZLE_128B)) {
    return cudaErrorInvalidValue;
  }
  static std::atomic<unsigned long long> attr_done{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = (dev >= 0 && dev < 64) ? 1ull << dev : 0ull;
  if (bit == 0 || (attr_done.load(std::memory_order_acquire) & bit) == 0) {
    const cudaError_t e = cudaFuncSetAttribute(
        gemm_w8t2_kernel<kBT>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    if (e != cudaSuccess) return e;
    attr_done.fetch_or(bit, std::memory_order_release);
  }
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int tiles = ((m + kBT - 1) / kBT) * ((n + 2 * kRows - 1) / (2 * kRows));
  const int pairs = sms / 2;
  const int clusters = tiles < pairs ? tiles : pairs;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * clusters);
  cfg.blockDim = dim3(C::kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, gemm_w8t2_kernel<kBT>, tx, tq,
                            reinterpret_cast<const uint16_t*>(scales), bias, output, m, n, k,
                            ldc, static_cast<const unsigned char*>(packed));
}

// ===================================================================
// Short prompts, few weight tiles: K split across a thread-block cluster.
//
// With <= 128 tokens and a narrow matrix (896 or 1152 outputs: 7-9 weight
// tiles) the kernels above keep only 7-9 SMs busy, each walking all of K.
// Here a cluster of S CTAs (S <= 8) shares one weight tile: CTA r of the
// cluster runs k-blocks [r*nkb/S, (r+1)*nkb/S) through the same
// TMA -> dequantise -> TMEM -> tcgen05.mma pipeline (single tile, single
// accumulator), parks its FP32 partial D [kBT tokens x 128 features] in its
// own shared memory, and after a cluster barrier CTA r adds, for its slice
// of the tokens, the S partials in rank order 0..S-1 read through
// distributed shared memory (ld.shared::cluster), then adds the bias and
// stores BF16.  One launch, no global scratch, deterministic; a different
// FP32 summation order from the unsplit kernels (fast order only).
// Every wait is bounded (2 s).
// ===================================================================
template <int kBT, bool kW16>
struct CfgS {
  static constexpr int kSub = 2;
  static constexpr int kKS = kBK * kSub;                  // K per stage
  static constexpr int kDqWarps = kW16 ? 0 : 8;
  static constexpr int kXSub = kBT * kBK * 2;
  static constexpr int kXBytes = kSub * kXSub;
  static constexpr int kWSub = kRows * kBK * 2;
  static constexpr int kQBytes = kW16 ? kSub * kWSub : kRows * kKS;
  static constexpr int kStageBytes = kXBytes + kQBytes;
  static constexpr int kRedBytes = kBT * kRows * 4;       // FP32 partial [tok][feat]
  static constexpr int kStages = 3 * kStageBytes + kRedBytes <= 216 * 1024 ? 3 : 2;
  static constexpr int kACols = kKS / 2;
  static constexpr int kAStages = kW16 ? 1 : 2;
  static constexpr int kACol0 = kBT;
  static constexpr int kTmemCols = 256;                   // kBT + 2 x 64 <= 256
  static constexpr int kThreads = (8 + kDqWarps) * 32;
  static constexpr int kSmemBytes = kStages * kStageBytes + kRedBytes + 512 + 1024;
  static_assert(kBT == 32 || kBT == 64 || kBT == 128, "token tile");
  static_assert(kW16 || kBT + kAStages * kACols <= kTmemCols, "TMEM columns");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory");
};

template <int kBT, bool kW16>
__global__ void __launch_bounds__(CfgS<kBT, kW16>::kThreads, 1)
gemm_w8t_split_kernel(const __grid_constant__ CUtensorMap tmap_x,
                      const __grid_constant__ CUtensorMap tmap_q,
                      const uint16_t* __restrict__ scales, const bf16* __restrict__ bias,
                      bf16* __restrict__ out, int m, int n, int k, int ldc) {
  using C = CfgS<kBT, kW16>;
  extern __shared__ __align__(1024) unsigned char smem_raws[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raws) + 1023) & ~uintptr_t(1023));
  float* red = reinterpret_cast<float*>(smem + C::kStages * C::kStageBytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<unsigned char*>(red) +
                                               C::kRedBytes);
  const uint32_t bar_full = smem_u32(bars);
  const uint32_t bar_empty = bar_full + 8 * C::kStages;
  const uint32_t bar_afull = bar_empty + 8 * C::kStages;
  const uint32_t bar_aempty = bar_afull + 8 * C::kAStages;
  const uint32_t bar_acc = bar_aempty + 8 * C::kAStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * C::kStages + 2 * C::kAStages + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int splits = int(gridDim.x);          // = cluster size
  const int rank = int(cluster_ctarank());
  const int nb = int(blockIdx.y), mb = int(blockIdx.z);
  const int num_kb = (k + C::kKS - 1) / C::kKS;
  const int kb0 = rank * num_kb / splits, kb1 = (rank + 1) * num_kb / splits;
  const int groups = (k + 63) / 64;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1 + C::kDqWarps);
    }
    for (int a = 0; a < C::kAStages; ++a) {
      mbar_init(bar_afull + 8 * a, C::kDqWarps > 0 ? C::kDqWarps : 1);
      mbar_init(bar_aempty + 8 * a, 1);
    }
    mbar_init(bar_acc, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(C::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_launch_dependents();
  pdl_wait_primary();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!wait_t(bar_empty + 8 * stage, phase ^ 1, abort_flag, B200_DEVICE_TIMEOUT_PIPELINE))
          break;
        unsigned char* st = smem + stage * C::kStageBytes;
        const uint32_t fb = bar_full + 8 * stage;
        mbar_arrive_expect_tx(fb, C::kStageBytes);
#pragma unroll
        for (int sub = 0; sub < C::kSub; ++sub) {
          tma_load_2d(smem_u32(st + sub * C::kXSub), &tmap_x, kb * C::kKS + sub * kBK,
                      mb * kBT, fb);
          if constexpr (kW16) {
            tma_load_2d(smem_u32(st + C::kXBytes + sub * C::kWSub), &tmap_q,
                        kb * C::kKS + sub * kBK, nb * kRows, fb);
          }
        }
        if constexpr (!kW16) {
          tma_load_2d(smem_u32(st + C::kXBytes), &tmap_q, kb * C::kKS, nb * kRows, fb);
        }
        if (++stage == C::kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(128, kBT);
      int stage = 0, aslot = 0;
      uint32_t phase = 0, aphase = 0;
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!wait_t(kW16 ? bar_full + 8 * stage : bar_afull + 8 * aslot, kW16 ? phase : aphase,
                    abort_flag, B200_DEVICE_TIMEOUT_PIPELINE)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t x_addr = smem_u32(smem + stage * C::kStageBytes);
        const uint32_t acc = (kb > kb0) ? 1u : 0u;
        if constexpr (kW16) {
          const uint32_t w_addr = x_addr + C::kXBytes;
#pragma unroll
          for (int kk = 0; kk < C::kKS / 16; ++kk) {
            mma_bf16(tmem_base, desc_sw128(w_addr + (kk >> 2) * C::kWSub + (kk & 3) * 32),
                     desc_sw128(x_addr + (kk >> 2) * C::kXSub + (kk & 3) * 32), idesc,
                     (acc || kk > 0) ? 1u : 0u);
          }
          mma_commit(bar_empty + 8 * stage);
        } else {
          const uint32_t a_addr = tmem_base + uint32_t(C::kACol0 + aslot * C::kACols);
#pragma unroll
          for (int kk = 0; kk < C::kKS / 16; ++kk) {
            mma_bf16_ta(tmem_base, a_addr + uint32_t(kk * 8),
                        desc_sw128(x_addr + (kk >> 2) * C::kXSub + (kk & 3) * 32), idesc,
                        (acc || kk > 0) ? 1u : 0u);
          }
          mma_commit(bar_empty + 8 * stage);
          mma_commit(bar_aempty + 8 * aslot);
        }
        if (++stage == C::kStages) {
          stage = 0;
          phase ^= 1;
        }
        if (++aslot == C::kAStages) {
          aslot = 0;
          aphase ^= 1;
        }
      }
      if (ok) mma_commit(bar_acc);
    }
  } else if (warp >= 4 && warp < 8) {
    // ---------------------- partial D -> this CTA's shared memory [tok][feat]
    const int q = warp & 3;
    const bool ok = __all_sync(0xffffffffu,
                               wait_t(bar_acc, 0, abort_flag, B200_DEVICE_TIMEOUT_ACCUM));
    tc_fence_after();
#pragma unroll 1
    for (int c0 = 0; c0 < kBT; c0 += 16) {
      uint32_t r[16];
      if (ok) {
        tmem_ld16(tmem_base + (uint32_t(q * 32) << 16) + uint32_t(c0), r);
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) r[j] = 0u;
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) red[(c0 + j) * kRows + q * 32 + lane] = __uint_as_float(r[j]);
    }
    tc_fence_before();
  } else if (!kW16 && warp >= 8) {
    // ---------------------------------------------------------- dequantiser
    const int dw = warp - 8;
    const int quarter = dw & 3;
    const int part = dw >> 2;
    const int rl = quarter * 32 + lane;
    const uint32_t t_lane = uint32_t(quarter * 32) << 16;
    const int sw = rl & 7;
    constexpr int kChunks = 4;
    const int row = nb * kRows + rl;
    const bool srow_ok = row < n;
    const uint16_t* srow = scales + size_t(srow_ok ? row : 0) * groups;
    int stage = 0, aslot = 0;
    uint32_t phase = 0, aphase = 0;
    for (int kb = kb0; kb < kb1; ++kb) {
      const int g = kb * 2 + part;
      const uint32_t sv = (srow_ok && g < groups) ? uint32_t(srow[g]) : 0u;
      if (!wait_t(bar_full + 8 * stage, phase, abort_flag, B200_DEVICE_TIMEOUT_PIPELINE)) break;
      const unsigned char* qt = smem + stage * C::kStageBytes + C::kXBytes + rl * C::kKS;
      uint4 c[kChunks];
#pragma unroll
      for (int j = 0; j < kChunks; ++j) {
        c[j] = *reinterpret_cast<const uint4*>(qt + (((part * kChunks + j) ^ sw) << 4));
      }
      const uint32_t s2bits = sv | (sv << 16);
      const bf162 s2 = *reinterpret_cast<const bf162*>(&s2bits);
      uint32_t v[8 * kChunks];
#pragma unroll
      for (int j = 0; j < kChunks; ++j) {
        dq4(c[j].x, s2, v + 8 * j + 0);
        dq4(c[j].y, s2, v + 8 * j + 2);
        dq4(c[j].z, s2, v + 8 * j + 4);
        dq4(c[j].w, s2, v + 8 * j + 6);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_empty + 8 * stage);
      if (!wait_t(bar_aempty + 8 * aslot, aphase ^ 1, abort_flag, B200_DEVICE_TIMEOUT_PIPELINE))
        break;
      tc_fence_after();
      const uint32_t ta = tmem_base + t_lane +
                          uint32_t(C::kACol0 + aslot * C::kACols + part * (C::kACols / 2));
#pragma unroll
      for (int j = 0; j < kChunks / 2; ++j) tmem_st16(ta + 16 * j, v + 16 * j);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_afull + 8 * aslot);
      if (++stage == C::kStages) {
        stage = 0;
        phase ^= 1;
      }
      if (++aslot == C::kAStages) {
        aslot = 0;
        aphase ^= 1;
      }
    }
  }

  // ------------------------------ fixed-order reduction across the cluster
  cluster_sync_all();  // every CTA's partial is in its shared memory
  {
    const int t0 = rank * kBT / splits, t1 = (rank + 1) * kBT / splits;
    const uint32_t red_local = smem_u32(red);
    for (int idx = int(threadIdx.x); idx < (t1 - t0) * kRows; idx += C::kThreads) {
      const int t = t0 + idx / kRows, f = idx % kRows;
      const uint32_t off = uint32_t((t * kRows + f) * 4);
      float sum = 0.0f;
      for (int j = 0; j < splits; ++j) {
        float v;
        asm volatile("ld.shared::cluster.f32 %0, [%1];"
                     : "=f"(v)
                     : "r"(map_to_rank(red_local, uint32_t(j)) + off)
                     : "memory");
        sum += v;
      }
      const int feat = nb * kRows + f, tok = mb * kBT + t;
      if (tok < m && feat < n) {
        if (bias != nullptr) sum += __bfloat162float(bias[feat]);
        out[size_t(tok) * ldc + feat] = __float2bfloat16_rn(sum);
      }
    }
  }
  cluster_sync_all();  // no CTA leaves while another still reads its partial
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(C::kTmemCols)
                 : "memory");
  }
}

template <int kBT, bool kW16>
cudaError_t launch_split_bt(const void* weight, const bf16* scales, const bf16* bias,
                            const bf16* input, bf16* output, int m, int n, int k, int ldc,
                            int splits, cudaStream_t stream) {
  using C = CfgS<kBT, kW16>;
  CUtensorMap tx, tq;
  if (!encode_tmap_2d(&tx, input, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, k, m, kBK, kBT,
                      CU_TENSOR_MAP_SWIZZLE_128B) ||
      !(kW16 ? encode_tmap_2d(&tq, weight, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, k, n, kBK,
                              kRows, CU_TENSOR_MAP_SWIZZLE_128B)
             : encode_tmap_2d(&tq, weight, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, k, n, C::kKS,
                              kRows, CU_TENSOR_MAP_SWIZZLE_128B))) {
    return cudaErrorInvalidValue;
  }
  static std::atomic<unsigned long long> attr_done{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = (dev >= 0 && dev < 64) ? 1ull << dev : 0ull;
  if (bit == 0 || (attr_done.load(std::memory_order_acquire) & bit) == 0) {
    const cudaError_t e = cudaFuncSetAttribute(gemm_w8t_split_kernel<kBT, kW16>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               C::kSmemBytes);
    if (e != cudaSuccess) return e;
    attr_done.fetch_or(bit, std::memory_order_release);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(splits, (n + kRows - 1) / kRows, (m + kBT - 1) / kBT);
  cfg.blockDim = dim3(C::kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  // A cluster of `splits` CTAs must fit on the device (checked once per
  // device and cluster size); otherwise the caller takes the unsplit kernel
  // instead of a launch that would fail.
  static std::atomic<int> fits[64][9];  // 0 unknown, 1 fits, 2 does not
  if (dev >= 0 && dev < 64 && splits <= 8) {
    int f = fits[dev][splits].load(std::memory_order_relaxed);
    if (f == 0) {
      int clusters = 0;
      const cudaError_t e = cudaOccupancyMaxActiveClusters(
          &clusters, gemm_w8t_split_kernel<kBT, kW16>, &cfg);
      if (e != cudaSuccess) cudaGetLastError();
      f = (e == cudaSuccess && clusters >= 1) ? 1 : 2;
      fits[dev][splits].store(f, std::memory_order_relaxed);
    }
    if (f == 2) return cudaErrorNotSupported;
  }
  return cudaLaunchKernelEx(&cfg, gemm_w8t_split_kernel<kBT, kW16>, tx, tq,
                            reinterpret_cast<const uint16_t*>(scales), bias, output, m, n, k,
                            ldc);
}

}  // namespace

bool gemm_w8t_supported(const void* weight, const void* input, const void* output, int m,
                        int n, int k) {
  return m > 0 && n > 0 && k > 0 && k % 16 == 0 &&
         (reinterpret_cast<uintptr_t>(weight) & 15u) == 0 &&
         (reinterpret_cast<uintptr_t>(input) & 15u) == 0 && output != nullptr;
}

cudaError_t launch_gemm_w8t(const void* weight, const bf16* scales, const bf16* bias,
                            const bf16* input, bf16* output, int m, int n, int k, int ldc,
                            cudaStream_t stream, const void* packed) {
  // Tile shape: tokens per tile x quantisation groups per stage
  // (B200_W8T_CFG=192x2 | 192x1 | 160x2 | 128x2 | 128x1 | 96x2 | 64x2 | 32x2 | p192 | p128
  // overrides, for
  // tuning; 160x2 leaves TMEM room for three A slots, 96x2 for five; 64x2 and
  // 32x2 for short prompts).
  const char* cfg = getenv("B200_W8T_CFG");
  if (cfg != nullptr && (packed == nullptr || !strstr(cfg, "x1"))) {
    if (!strcmp(cfg, "192x1")) return launch_bt<192, 1>(weight, scales, bias, input, output, m, n, k, ldc, stream);
    if (!strcmp(cfg, "128x1")) return launch_bt<128, 1>(weight, scales, bias, input, output, m, n, k, ldc, stream);
    if (!strcmp(cfg, "128x2")) return launch_bt<128, 2>(weight, scales, bias, input, output, m, n, k, ldc, stream, packed);
    if (!strcmp(cfg, "160x2")) return launch_bt<160, 2>(weight, scales, bias, input, output, m, n, k, ldc, stream, packed);
    if (!strcmp(cfg, "96x2")) return launch_bt<96, 2>(weight, scales, bias, input, output, m, n, k, ldc, stream, packed);
    if (!strcmp(cfg, "64x2")) return launch_bt<64, 2>(weight, scales, bias, input, output, m, n, k, ldc, stream, packed);
    if (!strcmp(cfg, "32x2")) return launch_bt<32, 2>(weight, scales, bias, input, output, m, n, k, ldc, stream, packed);
    if (!strcmp(cfg, "p192")) return launch_pair_bt<192>(weight, scales, bias, input, output, m, n, k, ldc, stream, packed);
    if (!strcmp(cfg, "p128")) return launch_pair_bt<128>(weight, scales, bias, input, output, m, n, k, ldc, stream, packed);
  }
  // Short prompts: the smallest token tile that covers them (no padding of
  // the MMA's N to 192).
  if (m <= 32) return launch_bt<32, 2>(weight, scales, bias, input, output, m, n, k, ldc, stream, packed);
  if (m <= 64) return launch_bt<64, 2>(weight, scales, bias, input, output, m, n, k, ldc, stream, packed);
  // 65..128 tokens: two 64-token tiles when the weight tiles alone leave
  // most SMs idle (128 x 896 -> 4864: 10.25 -> 8.62 us).
  if (m <= 128 && (n + kRows - 1) / kRows < 74) {
    return launch_bt<64, 2>(weight, scales, bias, input, output, m, n, k, ldc, stream, packed);
  }
  if (m <= 128) return launch_bt<128, 2>(weight, scales, bias, input, output, m, n, k, ldc, stream, packed);
  // Long prompts up to 2^29 outputs: the CTA-pair form, measured 2-6% faster
  // (e.g. 8192 x 4864 -> 896: 92.4 -> 87.3 us); 10% slower at 8192 x 896 ->
  // 151936, which stays on the one-SM form.
  if (m >= 1024 && double(m) * double(n) < double(1 << 29)) {
    return launch_pair_bt<192>(weight, scales, bias, input, output, m, n, k, ldc, stream, packed);
  }
  // 192-token tiles unless 128-token tiles pad noticeably less (256 tokens
  // pad to 384 with 192: 128-token tiles measured 99 vs 128 us on 896 ->
  // 151936).
  const int pad128 = (m + 127) / 128 * 128, pad192 = (m + 191) / 192 * 192;
  if (double(pad128) < 0.85 * double(pad192)) {
    return launch_bt<128, 2>(weight, scales, bias, input, output, m, n, k, ldc, stream, packed);
  }
  return launch_bt<192, 2>(weight, scales, bias, input, output, m, n, k, ldc, stream, packed);
}

// BF16 weights in the same transposed form (weights the MMA's M side from
// shared memory, tokens its N side): for prompts of <= 128 tokens, whose
// token tile is then 32 / 64 / 128 instead of padding to 128 tokens x a
// narrow weight tile.
cudaError_t launch_gemm_w16t(const bf16* weight, const bf16* bias, const bf16* input,
                             bf16* output, int m, int n, int k, int ldc, cudaStream_t stream) {
  if (m <= 32) return launch_bt<32, 2, true>(weight, nullptr, bias, input, output, m, n, k, ldc, stream);
  if (m <= 64) return launch_bt<64, 2, true>(weight, nullptr, bias, input, output, m, n, k, ldc, stream);
  return launch_bt<128, 2, true>(weight, nullptr, bias, input, output, m, n, k, ldc, stream);
}

// Cluster split-K for short prompts on narrow matrices (fast order).
// Returns cudaErrorNotSupported when the shape does not qualify: <= 512
// tokens (<= 128 unless K is long), at most 37 output tiles (a quarter of the SMs), at least two
// 128-wide k-blocks per split, and a shape where it measured faster: long K
// (32 x 4864 -> 896: W8A16 25.8 -> 7.3 us, BF16 18.5 -> 6.0 us; 128 tokens:
// 26.5 -> 9.7 / 21.0 -> 9.8 us, ahead of the reserved-buffer split) or
// W8A16 at <= 32 tokens (896 -> 896: 7.5 -> 6.3 us).  At K = 896 with more
// tokens, or in BF16, the unsplit kernels stay faster.
cudaError_t launch_gemm_cluster_split(bool w8, const void* weight, const bf16* scales,
                                      const bf16* bias, const bf16* input, bf16* output,
                                      int m, int n, int k, int ldc, cudaStream_t stream) {
  if (m <= 0 || m > 512) return cudaErrorNotSupported;
  if (!(k >= 2048 || (w8 && m <= 32))) return cudaErrorNotSupported;
  const int bt = m <= 32 ? 32 : (m <= 64 ? 64 : 128);
  const int tiles = ((n + kRows - 1) / kRows) * ((m + bt - 1) / bt);
  const int num_kb = (k + 127) / 128;
  if (tiles > 37) return cudaErrorNotSupported;
  // 129..512 tokens (measured): long K with room for ~8 splits (256 x 4864 ->
  // 896: 31.0 -> 10.2 us; 512 x 4864 -> 128: 30.8 -> 9.5 us), or W8A16 with
  // K >= 4096 (512 x 4864 -> 896: 31.2 -> 24.1 us); fewer splits or K = 2048
  // measured slower.
  if (m > 128 && !(k >= 2048 && (tiles <= 18 || (w8 && k >= 4096)))) {
    return cudaErrorNotSupported;
  }
  int sms = 148;
  int dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int splits = sms / tiles;
  if (splits > 8) splits = 8;
  if (splits > num_kb / 2) splits = num_kb / 2;
  if (splits < 2) return cudaErrorNotSupported;
  if (w8) {
    if (bt == 32) return launch_split_bt<32, false>(weight, scales, bias, input, output, m, n, k, ldc, splits, stream);
    if (bt == 64) return launch_split_bt<64, false>(weight, scales, bias, input, output, m, n, k, ldc, splits, stream);
    return launch_split_bt<128, false>(weight, scales, bias, input, output, m, n, k, ldc, splits, stream);
  }
  if (bt == 32) return launch_split_bt<32, true>(weight, nullptr, bias, input, output, m, n, k, ldc, splits, stream);
  if (bt == 64) return launch_split_bt<64, true>(weight, nullptr, bias, input, output, m, n, k, ldc, splits, stream);
  return launch_split_bt<128, true>(weight, nullptr, bias, input, output, m, n, k, ldc, splits, stream);
}

// ---------------------------------------------------------- pre-packing
// Packed W8A16 weights: [2 ceil(N/256)][ceil(K/128)] tiles of 16 KB; tile
// (tn, tk) holds rows tn*128.. and K values tk*128.. exactly as the kernels'
// shared memory holds them after a 128-byte-swizzled TMA load (row r at
// r * 128, its 16-byte chunk c at position c ^ (r & 7)), zero outside the
// matrix.  One 1-D bulk copy then brings a tile: contiguous DRAM reads
// instead of a box of 128 rows x 128 bytes strided by K.
__global__ void __launch_bounds__(256)
pack_w8a16_kernel(const int8_t* __restrict__ q, int n, int k, int tiles_k,
                  uint4* __restrict__ out, size_t chunks) {
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < chunks;
       i += size_t(gridDim.x) * blockDim.x) {
    const size_t tile = i >> 10;  // 1024 chunks of 16 bytes per tile
    const int within = int(i & 1023);
    const int r = within >> 3, pos = within & 7;
    const int c = pos ^ (r & 7);
    const int tn = int(tile / tiles_k), tk = int(tile % tiles_k);
    const int row = tn * kRows + r;
    const int col = tk * 128 + c * 16;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (row < n && col < k) v = *reinterpret_cast<const uint4*>(q + size_t(row) * k + col);
    out[i] = v;
  }
}

// The tile count along N is rounded up to even: the CTA-pair kernel reads
// tiles 2 nb and 2 nb + 1 (the padding tiles are zero).
size_t w8a16_packed_bytes(int n, int k) {
  if (n <= 0 || k <= 0) return 0;
  const size_t tiles_n = size_t((n + 2 * kRows - 1) / (2 * kRows)) * 2;
  return tiles_n * size_t((k + 127) / 128) * 16384;
}

cudaError_t launch_pack_w8a16(const int8_t* q, int n, int k, void* packed,
                              cudaStream_t stream) {
  const size_t chunks = w8a16_packed_bytes(n, k) / 16;
  if (chunks == 0) return cudaSuccess;
  size_t grid = (chunks + 255) / 256;
  if (grid > 148 * 16) grid = 148 * 16;
  pack_w8a16_kernel<<<unsigned(grid), 256, 0, stream>>>(q, n, k, (k + 127) / 128,
                                                        static_cast<uint4*>(packed), chunks);
  return cudaGetLastError();
}

}  // namespace b200
