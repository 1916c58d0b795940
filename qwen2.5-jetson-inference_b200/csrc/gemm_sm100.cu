// Prefill GEMM on the 5th-generation tensor cores (sm_100a):
//   Y[M,N] = bf16( X[M,K] . W[N,K]^T + b[N] ),  FP32 accumulation in TMEM.
//
// Replaces the reference's WMMA GEMMs gemm_bf16 / gemm_w8a16
// (src/cuda/kernels.cu:605-951, 1096-1322, dispatch 1600-1684).
//
// Structure (one persistent CTA per SM, warp-specialised):
//   warp 0        TMA producer: X tile(s) [128 x 64] BF16 (128-byte swizzle)
//                 and the W tile [BN x 64] (BF16 swizzled, or raw INT8)
//                 into a ring of shared-memory stages (mbarrier complete_tx).
//   warp 1        TMEM allocator and the single-thread tcgen05.mma issuer:
//                 MSUB x (M=128, N=BN, K=16) MMAs per 16-wide k step, FP32
//                 accumulators in TMEM, double-buffered across tiles;
//                 tcgen05.commit releases smem stages and hands finished
//                 accumulators to the epilogue.
//   warps 4..7    epilogue: tcgen05.ld 32 columns at a time, + bias, BF16
//                 round-to-nearest-even, store.
//   warps 8..15   (W8A16 only) dequantisers: raw INT8 tile -> bf16(q * s)
//                 written straight into the 128-byte-swizzled K-major layout
//                 the MMA reads, then fence.proxy.async and an mbarrier
//                 arrive.  One BK=64 k-block is exactly one quantisation
//                 group, so each W row needs one scale per stage.
//
// The BF16 rounding of q*s matches the reference's tensor-core GEMM
// (src/cuda/kernels.cu:1084-1092): the product of an int8 and a BF16 scale
// is exact in FP32 and fma.rn.bf16x2(q, s, -0) rounds it once.
//
// Every mbarrier wait is bounded (kWaitTimeoutNs); on expiry the CTA records
// B200_DEVICE_TIMEOUT_* in g_device_status, raises a shared abort flag so
// the other roles stop waiting, frees its TMEM and returns.
//
// No TMA multicast is used (this kernel also runs on every rank of the
// column-sharded GEMM).

#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <cstring>
#include <atomic>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace b200 {

__device__ int g_device_status = 0;

cudaError_t read_device_status(int* value, bool clear) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return e;
  e = cudaMemcpyFromSymbol(value, g_device_status, sizeof(int));
  if (e != cudaSuccess) return e;
  if (clear) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int));
  }
  return e;
}

namespace {

constexpr int kBK = 64;                    // K per stage = one W8 group

// Bounded wait that records into this file's device status word.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity,
                                          volatile int* abort_flag,
                                          int error_code) {
  return mbar_wait_bounded(bar, parity, abort_flag, error_code,
                           &g_device_status);
}

// --------------------------------------------------------------- the kernel
template <bool kW8, int kMSub, int kBN>
struct Cfg {
  static constexpr int kBM = 128 * kMSub;
  static constexpr int kABytes = 128 * kBK * 2;          // one 128-row sub-tile
  static constexpr int kBBytes = kBN * kBK * 2;          // BF16 B tile
  static constexpr int kQBytes = kW8 ? kBN * kBK : 0;    // raw INT8 B tile
  static constexpr int kStageBytes = kMSub * kABytes + kBBytes + kQBytes;
  static constexpr int kStages = (200 * 1024) / kStageBytes > 6
                                     ? 6
                                     : (200 * 1024) / kStageBytes;
  static constexpr int kAccCols = kMSub * kBN;           // fp32 columns / tile
  static constexpr int kAccBufs = 2 * kAccCols <= 512 ? 2 : 1;
  static constexpr int kTmemCols = kAccBufs * kAccCols;  // power of two
  static constexpr int kDqWarps = kW8 ? 8 : 0;
  static constexpr int kWarps = 8 + kDqWarps;
  static constexpr int kThreads = kWarps * 32;
  static constexpr int kTxBytes = kMSub * kABytes + (kW8 ? kQBytes : kBBytes);
  static constexpr int kBarrierBytes = 256;
  static constexpr int kSmemBytes = kStages * kStageBytes + kBarrierBytes + 1024;
  static_assert(kTmemCols == 32 || kTmemCols == 64 || kTmemCols == 128 ||
                    kTmemCols == 256 || kTmemCols == 512,
                "TMEM allocation must be a power of two >= 32");
  static_assert(kBN % 32 == 0 && kBN >= 32 && kBN <= 256, "bad BN");
};

struct TileIter {
  int tile, kb;
};

template <bool kW8, int kMSub, int kBN>
__global__ void __launch_bounds__(Cfg<kW8, kMSub, kBN>::kThreads, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_x,
               const __grid_constant__ CUtensorMap tmap_w,
               const bf16* __restrict__ scales, const bf16* __restrict__ bias,
               bf16* __restrict__ out, int m, int n, int k, int ldc,
               const PeerOuts peers, int a_rows, int kchunk,
               float* __restrict__ partial) {
  using C = Cfg<kW8, kMSub, kBN>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // 1024-byte alignment for the swizzle atoms.
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* stage_base = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
  // bars: full[S], dq_full[S], empty[S], acc_full[2], acc_empty[2]
  const uint32_t bar_full = smem_u32(bars);
  const uint32_t bar_dq = bar_full + 8 * C::kStages;
  const uint32_t bar_empty = bar_dq + 8 * C::kStages;
  const uint32_t bar_acc_full = bar_empty + 8 * C::kStages;
  const uint32_t bar_acc_empty = bar_acc_full + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * C::kStages + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (m + C::kBM - 1) / C::kBM;
  const int num_n = (n + kBN - 1) / kBN;
  const int num_tiles = num_m * num_n;
  // K split (grid z): this CTA walks K values [k_begin, k_begin + kchunk) and,
  // with `partial`, stores FP32 sums without bias into slab z of it.
  const int k_begin = int(blockIdx.z) * kchunk;
  const int k_len = k - k_begin < kchunk ? k - k_begin : kchunk;
  const int num_kb = (k_len + kBK - 1) / kBK;
  const int kb0 = k_begin / kBK;  // kchunk is a multiple of kBK
  const int groups = (k + 63) / 64;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_dq + 8 * s, C::kDqWarps > 0 ? C::kDqWarps * 32 : 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(bar_acc_full + 8 * a, 1);
      mbar_init(bar_acc_empty + 8 * a, 128);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile(
        "tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
            smem_u32(tmem_slot)),
        "r"(C::kTmemCols)
        : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::
                     : "memory");
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
          if (!mbar_wait(bar_empty + 8 * stage, phase ^ 1, abort_flag,
                         B200_DEVICE_TIMEOUT_PIPELINE))
            goto producer_done;
          unsigned char* st = stage_base + stage * C::kStageBytes;
          const uint32_t fb = bar_full + 8 * stage;
          // X rows per sub-tile: 128, or fewer for a short prompt (a_rows, the
          // TMA box height); the MMA's rows beyond them are never stored.
          mbar_arrive_expect_tx(fb, C::kTxBytes - kMSub * (128 - a_rows) * kBK * 2);
#pragma unroll
          for (int s = 0; s < kMSub; ++s) {
            tma_load_2d(smem_u32(st + s * C::kABytes), &tmap_x, (kb0 + kb) * kBK,
                        mb * C::kBM + s * 128, fb);
          }
          unsigned char* wdst = st + kMSub * C::kABytes + (kW8 ? C::kBBytes : 0);
          tma_load_2d(smem_u32(wdst), &tmap_w, (kb0 + kb) * kBK, nb * kBN, fb);
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
      constexpr uint32_t idesc = idesc_bf16(128, kBN);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++it) {
        const int buf = C::kAccBufs == 2 ? (it & 1) : 0;
        const uint32_t use = C::kAccBufs == 2 ? ((it >> 1) & 1) : (it & 1);
        if (!mbar_wait(bar_acc_empty + 8 * buf, use ^ 1, abort_flag,
                       B200_DEVICE_TIMEOUT_ACCUM))
          break;
        tc_fence_after();
        const uint32_t d_base = tmem_base + uint32_t(buf * C::kAccCols);
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          const uint32_t ready = kW8 ? bar_dq + 8 * stage : bar_full + 8 * stage;
          if (!mbar_wait(ready, phase, abort_flag, B200_DEVICE_TIMEOUT_PIPELINE)) {
            ok = false;
            break;
          }
          tc_fence_after();
          unsigned char* st = stage_base + stage * C::kStageBytes;
          const uint32_t b_addr = smem_u32(st + kMSub * C::kABytes);
#pragma unroll
          for (int s = 0; s < kMSub; ++s) {
            const uint32_t a_addr = smem_u32(st + s * C::kABytes);
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk) {
              mma_bf16(d_base + uint32_t(s * kBN), desc_sw128(a_addr + kk * 32),
                       desc_sw128(b_addr + kk * 32), idesc,
                       (kb > 0 || kk > 0) ? 1u : 0u);
            }
          }
          mma_commit(bar_empty + 8 * stage);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit(bar_acc_full + 8 * buf);
      }
    }
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter
    const bool vec_ok =
        (ldc % 8 == 0) && ((reinterpret_cast<uintptr_t>(out) & 15u) == 0);
    int it = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++it) {
      const int mb = tile % num_m;
      const int nb = tile / num_m;
      const int buf = C::kAccBufs == 2 ? (it & 1) : 0;
      const uint32_t use = C::kAccBufs == 2 ? ((it >> 1) & 1) : (it & 1);
      // Warp-uniform decision: tcgen05.ld needs every lane of the warp.
      const bool acc_ok = mbar_wait(bar_acc_full + 8 * buf, use, abort_flag,
                                    B200_DEVICE_TIMEOUT_ACCUM);
      if (!__all_sync(0xffffffffu, acc_ok)) break;
      tc_fence_after();
#pragma unroll 1
      for (int s = 0; s < kMSub; ++s) {
        const int row = mb * C::kBM + s * 128 + q * 32 + lane;
#pragma unroll 1
        for (int c0 = 0; c0 < kBN; c0 += 32) {
          uint32_t r[32];
          tmem_ld32(tmem_base + (uint32_t(q * 32) << 16) +
                        uint32_t(buf * C::kAccCols + s * kBN + c0),
                    r);
          const int col0 = nb * kBN + c0;
          if (partial != nullptr) {
            // K-split partial: FP32, no bias, slab blockIdx.z of [m][n]
            if (row < m) {
              float* pd = partial + (size_t(blockIdx.z) * m + row) * n + col0;
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                if (col0 + j < n) pd[j] = __uint_as_float(r[j]);
              }
            }
          } else if (row < m && col0 < n) {
            bf16* dst = out + size_t(row) * ldc + col0;
            if (vec_ok && col0 + 32 <= n) {
#pragma unroll
              for (int v = 0; v < 4; ++v) {
                uint32_t packed[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const int j = v * 8 + e * 2;
                  float f0 = __uint_as_float(r[j]);
                  float f1 = __uint_as_float(r[j + 1]);
                  if (bias) {
                    f0 += __bfloat162float(bias[col0 + j]);
                    f1 += __bfloat162float(bias[col0 + j + 1]);
                  }
                  const bf162 h = __floats2bfloat162_rn(f0, f1);
                  packed[e] = *reinterpret_cast<const uint32_t*>(&h);
                }
                const uint4 val = make_uint4(packed[0], packed[1], packed[2], packed[3]);
                reinterpret_cast<uint4*>(dst)[v] = val;
                for (int pi = 0; pi < peers.n; ++pi) {
                  reinterpret_cast<uint4*>(reinterpret_cast<char*>(dst) + peers.delta[pi])[v] = val;
                }
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                if (col0 + j < n) {
                  float f = __uint_as_float(r[j]);
                  if (bias) f += __bfloat162float(bias[col0 + j]);
                  const bf16 hv = __float2bfloat16_rn(f);
                  dst[j] = hv;
                  for (int pi = 0; pi < peers.n; ++pi) {
                    reinterpret_cast<bf16*>(reinterpret_cast<char*>(dst) + peers.delta[pi])[j] = hv;
                  }
                }
              }
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(bar_acc_empty + 8 * buf);
    }
    // Stores into other GPUs' memory are made visible system-wide before
    // the kernel completes.
    if (peers.n > 0) __threadfence_system();
  } else if (warp >= 8) {
    // ---------------------------------------------------------- dequantiser
    if constexpr (kW8) {
    const int dt = threadIdx.x - 8 * 32;        // 0 .. 255
    constexpr int kItems = kBN * 4;             // (row, 16-byte chunk) pairs
    constexpr int kPerThread = kItems / (C::kDqWarps * 32);
    static_assert(kItems % (C::kDqWarps * 32) == 0, "dequant split");
    // Scales are read from global memory kAhead stages before they are
    // needed (a register ring indexed by the unrolled loop position, so no
    // load result is moved before it arrives): the L2 latency of the scale
    // reads stays off the dequant critical path.
    constexpr int kAhead = 4;
    const uint16_t* sbits = reinterpret_cast<const uint16_t*>(scales);
    auto load_scales = [&](int tile, int kb, uint32_t* out) {
      const int nb = tile / num_m;
#pragma unroll
      for (int p = 0; p < kPerThread; ++p) {
        const int item = dt + p * (C::kDqWarps * 32);
        const int row = nb * kBN + (item >> 2);
        const uint32_t v =
            (tile < num_tiles && row < n) ? sbits[size_t(row) * groups + kb0 + kb] : 0u;
        out[p] = v | (v << 16);
      }
    };
    int pf_tile = blockIdx.x, pf_kb = 0;
    uint32_t sq[kAhead][kPerThread];
#pragma unroll
    for (int d = 0; d < kAhead; ++d) {
      load_scales(pf_tile, pf_kb, sq[d]);
      if (++pf_kb == num_kb) {
        pf_kb = 0;
        pf_tile += gridDim.x;
      }
    }
    int stage = 0;
    uint32_t phase = 0;
    int tile = blockIdx.x, kb = 0;
    const bf162 neg0 = __halves2bfloat162(__ushort_as_bfloat16(0x8000),
                                          __ushort_as_bfloat16(0x8000));
    while (true) {
#pragma unroll
      for (int d = 0; d < kAhead; ++d) {
        if (tile >= num_tiles) goto dequant_done;
        if (!mbar_wait(bar_full + 8 * stage, phase, abort_flag,
                       B200_DEVICE_TIMEOUT_PIPELINE))
          goto dequant_done;
        unsigned char* st = stage_base + stage * C::kStageBytes;
        unsigned char* bt = st + kMSub * C::kABytes;
        const unsigned char* qt = bt + C::kBBytes;
#pragma unroll
        for (int p = 0; p < kPerThread; ++p) {
          const int item = dt + p * (C::kDqWarps * 32);
          const int r = item >> 2;
          const int j = item & 3;
          const uint4 raw = *reinterpret_cast<const uint4*>(qt + r * kBK + j * 16);
          const uint32_t s2bits = sq[d][p];
          const bf162 s2 = *reinterpret_cast<const bf162*>(&s2bits);
          uint32_t outw[8];
          const uint32_t words[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
          for (int wi = 0; wi < 4; ++wi) {
            const uint32_t b = words[wi] ^ 0x80808080u;
            const uint32_t f0 = __float_as_uint(s8_to_f32_biased<0>(b));
            const uint32_t f1 = __float_as_uint(s8_to_f32_biased<1>(b));
            const uint32_t f2 = __float_as_uint(s8_to_f32_biased<2>(b));
            const uint32_t f3 = __float_as_uint(s8_to_f32_biased<3>(b));
            // q has <= 8 significant bits, so its BF16 is the top half.
            uint32_t q01 = __byte_perm(f0, f1, 0x7632);
            uint32_t q23 = __byte_perm(f2, f3, 0x7632);
            bf162 d01 = __hfma2(*reinterpret_cast<bf162*>(&q01), s2, neg0);
            bf162 d23 = __hfma2(*reinterpret_cast<bf162*>(&q23), s2, neg0);
            outw[2 * wi] = *reinterpret_cast<uint32_t*>(&d01);
            outw[2 * wi + 1] = *reinterpret_cast<uint32_t*>(&d23);
          }
          // 16 BF16 = 16-byte chunks 2j and 2j+1 of row r, 128B-swizzled.
          unsigned char* rowp = bt + (r >> 3) * 1024 + (r & 7) * 128;
          const int c0 = (2 * j) ^ (r & 7);
          const int c1 = (2 * j + 1) ^ (r & 7);
          *reinterpret_cast<uint4*>(rowp + c0 * 16) =
              make_uint4(outw[0], outw[1], outw[2], outw[3]);
          *reinterpret_cast<uint4*>(rowp + c1 * 16) =
              make_uint4(outw[4], outw[5], outw[6], outw[7]);
        }
        fence_proxy_async_smem();
        mbar_arrive(bar_dq + 8 * stage);
        if (++stage == C::kStages) {
          stage = 0;
          phase ^= 1;
        }
        // Refill this ring slot kAhead stages ahead.
        load_scales(pf_tile, pf_kb, sq[d]);
        if (++pf_kb == num_kb) {
          pf_kb = 0;
          pf_tile += gridDim.x;
        }
        if (++kb == num_kb) {
          kb = 0;
          tile += gridDim.x;
        }
      }
    }
  dequant_done:;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(
                     tmem_base),
                 "r"(C::kTmemCols)
                 : "memory");
  }
}

// ===================================================================
// CTA-pair (cta_group::2) GEMM: one 256 x kBN2 output tile per pair of SMs.
//
// The two CTAs of a cluster each load 128 rows of X and half (kBN2/2 rows)
// of the W tile; the leader CTA (rank 0) issues one
// tcgen05.mma.cta_group::2 (M=256, N=kBN2, K=16) per k step, which reads A
// from each CTA's own shared memory and B from both halves, and writes each
// CTA's 128 output rows into that CTA's TMEM.  Per SM this halves the
// shared-memory traffic of the W operand (loaded once per pair, read once)
// compared with a one-SM 128 x kBN2 tile -- shared-memory bandwidth
// (TMA writes + MMA operand reads) is what bounds the one-SM kernel.
//
// Synchronisation (barrier offsets are identical in both CTAs):
//   full[s]   leader; X (and BF16 W) tiles of BOTH CTAs complete_tx here
//             (the .cta_group::2 TMA form routes the peer's bytes to it);
//   fullq[s]  each CTA, its raw INT8 W half (W8A16);
//   empty[s]  each CTA; the leader's tcgen05.commit multicasts to both;
//   W8A16 only: the dequantised W halves live in a separate 3-slot ring,
//   dq[d]     leader; one arrival per CTA after its dequant threads meet
//             on a named barrier (the peer's arrival is remote);
//   dq_empty[d] each CTA (commit multicast) -- so the TMA ring of X and raw
//             INT8 tiles can run 6 stages ahead of the dequant hand-off;
//   acc_full  each CTA (commit multicast); acc_empty leader, one arrival
//             per CTA after its four epilogue warps meet.
// No TMA multicast is used.  All waits are bounded as in the one-SM kernel.
// ===================================================================
// Bounded wait with cluster-scope acquire (arrivals come from the peer CTA).
__device__ __forceinline__ bool mbar_wait_cl(uint32_t bar, uint32_t parity,
                                             volatile int* abort_flag, int code) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  while (true) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if (*abort_flag) return false;
    if (global_timer_ns() - start > kWaitTimeoutNs) {
      *abort_flag = 1;
      atomicCAS(&g_device_status, 0, code);
      return false;
    }
  }
}
template <bool kW8>
struct Cfg2 {
  static constexpr int kBN = 256;                 // pair tile N
  static constexpr int kHalf = kBN / 2;           // W rows per CTA
  static constexpr int kABytes = 128 * kBK * 2;   // 16 KB
  static constexpr int kBBytes = kHalf * kBK * 2; // 16 KB (BF16 half tile)
  static constexpr int kQBytes = kW8 ? kHalf * kBK : 0;
  // Raw ring (TMA destination): X half + (BF16 W half | raw INT8 W half).
  static constexpr int kStageBytes = kABytes + (kW8 ? kQBytes : kBBytes);
  // INT8: a separate, shorter ring of dequantised W halves, so the TMA ring
  // runs deep ahead of the dequant -> MMA hand-off.
  static constexpr int kDqStages = kW8 ? 3 : 0;
  static constexpr int kDqBytes = kW8 ? kBBytes : 0;
  static constexpr int kRingBudget = 196 * 1024 - kDqStages * kDqBytes;
  static constexpr int kStages = kRingBudget / kStageBytes > 6 ? 6
                                                               : kRingBudget / kStageBytes;
  static constexpr int kAccCols = kBN;            // fp32 columns per buffer
  static constexpr int kTmemCols = 2 * kAccCols;  // 512
  static constexpr int kDqWarps = kW8 ? 8 : 0;
  static constexpr int kWarps = 8 + kDqWarps;
  static constexpr int kThreads = kWarps * 32;
  static constexpr int kSmemBytes =
      kStages * kStageBytes + kDqStages * kDqBytes + 512 + 1024;
};

template <bool kW8>
__global__ void __launch_bounds__(Cfg2<kW8>::kThreads, 1)
gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmap_x,
                const __grid_constant__ CUtensorMap tmap_w,
                const bf16* __restrict__ scales, const bf16* __restrict__ bias,
                bf16* __restrict__ out, int m, int n, int k, int ldc,
                const PeerOuts peers) {
  using C = Cfg2<kW8>;
  extern __shared__ __align__(1024) unsigned char smem_raw2[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw2) + 1023) & ~uintptr_t(1023));
  unsigned char* dq_ring = smem + C::kStages * C::kStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(dq_ring + C::kDqStages * C::kDqBytes);
  const uint32_t bar_full = smem_u32(bars);
  const uint32_t bar_fullq = bar_full + 8 * C::kStages;
  const uint32_t bar_empty = bar_fullq + 8 * C::kStages;
  const uint32_t bar_dq = bar_empty + 8 * C::kStages;          // [kDqStages]
  const uint32_t bar_dq_empty = bar_dq + 8 * C::kDqStages;     // [kDqStages]
  const uint32_t bar_acc_full = bar_dq_empty + 8 * C::kDqStages;
  const uint32_t bar_acc_empty = bar_acc_full + 16;
  uint32_t* tmem_slot =
      reinterpret_cast<uint32_t*>(bars + 3 * C::kStages + 2 * C::kDqStages + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster = blockIdx.x >> 1;
  const int num_clusters = gridDim.x >> 1;
  const int num_m = (m + 255) / 256;
  const int num_n = (n + C::kBN - 1) / C::kBN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (k + kBK - 1) / kBK;
  const int groups = (k + 63) / 64;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_fullq + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    for (int d = 0; d < C::kDqStages; ++d) {
      mbar_init(bar_dq + 8 * d, 2);        // one arrival per CTA
      mbar_init(bar_dq_empty + 8 * d, 1);  // leader's commit multicast
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(bar_acc_full + 8 * a, 1);
      mbar_init(bar_acc_empty + 8 * a, 2);  // one arrival per CTA
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile(
        "tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
            smem_u32(tmem_slot)),
        "r"(C::kTmemCols)
        : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();
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
      for (int tile = cluster; tile < num_tiles; tile += num_clusters) {
        const int mb = tile % num_m;
        const int nb = tile / num_m;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_cl(bar_empty + 8 * stage, phase ^ 1, abort_flag,
                            B200_DEVICE_TIMEOUT_PIPELINE))
            goto producer2_done;
          unsigned char* st = smem + stage * C::kStageBytes;
          const uint32_t fb = bar_full + 8 * stage;
          if (leader) {
            mbar_arrive_expect_tx(fb, 2 * (C::kABytes + (kW8 ? 0 : C::kBBytes)));
          }
          tma_load_2d_pair(smem_u32(st), &tmap_x, kb * kBK, mb * 256 + rank * 128, fb);
          const int wrow = nb * C::kBN + rank * C::kHalf;
          if constexpr (kW8) {
            const uint32_t qb = bar_fullq + 8 * stage;
            mbar_arrive_expect_tx(qb, C::kQBytes);
            tma_load_2d(smem_u32(st + C::kABytes), &tmap_w, kb * kBK, wrow, qb);
          } else {
            tma_load_2d_pair(smem_u32(st + C::kABytes), &tmap_w, kb * kBK, wrow, fb);
          }
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  producer2_done:;
  } else if (warp == 1) {
    // ------------------------------------------------------ MMA (leader)
    if (leader && lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(256, C::kBN);
      int stage = 0;
      uint32_t phase = 0;
      int dstage = 0;
      uint32_t dphase = 0;
      int it = 0;
      for (int tile = cluster; tile < num_tiles; tile += num_clusters, ++it) {
        const int buf = it & 1;
        const uint32_t use = (it >> 1) & 1;
        if (!mbar_wait_cl(bar_acc_empty + 8 * buf, use ^ 1, abort_flag,
                          B200_DEVICE_TIMEOUT_ACCUM))
          break;
        tc_fence_after();
        const uint32_t d_base = tmem_base + uint32_t(buf * C::kAccCols);
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_cl(bar_full + 8 * stage, phase, abort_flag,
                            B200_DEVICE_TIMEOUT_PIPELINE) ||
              (kW8 && !mbar_wait_cl(bar_dq + 8 * dstage, dphase, abort_flag,
                                    B200_DEVICE_TIMEOUT_PIPELINE))) {
            ok = false;
            break;
          }
          tc_fence_after();
          unsigned char* st = smem + stage * C::kStageBytes;
          const uint32_t a_addr = smem_u32(st);
          const uint32_t b_addr =
              kW8 ? smem_u32(dq_ring + dstage * C::kDqBytes) : smem_u32(st + C::kABytes);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            mma2_bf16(d_base, desc_sw128(a_addr + kk * 32), desc_sw128(b_addr + kk * 32),
                      idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          mma2_commit_both(bar_empty + 8 * stage);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
          if constexpr (kW8) {
            mma2_commit_both(bar_dq_empty + 8 * dstage);
            if (++dstage == C::kDqStages) {
              dstage = 0;
              dphase ^= 1;
            }
          }
        }
        if (!ok) break;
        mma2_commit_both(bar_acc_full + 8 * buf);
      }
    }
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const bool vec_ok = (ldc % 8 == 0) && ((reinterpret_cast<uintptr_t>(out) & 15u) == 0);
    const uint32_t acc_empty_leader = map_to_rank(bar_acc_empty, 0);
    int it = 0;
    for (int tile = cluster; tile < num_tiles; tile += num_clusters, ++it) {
      const int mb = tile % num_m;
      const int nb = tile / num_m;
      const int buf = it & 1;
      const uint32_t use = (it >> 1) & 1;
      // A failed wait does not leave the loop: every epilogue thread must
      // still meet the others at the named barrier below (a thread that left
      // would strand them); once the abort flag is up the remaining waits
      // fail at once and the work is skipped.  The decision is warp-uniform
      // because tcgen05.ld needs every lane of the warp.
      const bool acc_ok = __all_sync(
          0xffffffffu,
          mbar_wait_cl(bar_acc_full + 8 * buf, use, abort_flag, B200_DEVICE_TIMEOUT_ACCUM));
      tc_fence_after();
      const int row = mb * 256 + int(rank) * 128 + q * 32 + lane;
#pragma unroll 1
      for (int c0 = 0; acc_ok && c0 < C::kBN; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(tmem_base + (uint32_t(q * 32) << 16) + uint32_t(buf * C::kAccCols + c0), r);
        const int col0 = nb * C::kBN + c0;
        if (row < m && col0 < n) {
          bf16* dst = out + size_t(row) * ldc + col0;
          if (vec_ok && col0 + 32 <= n) {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint32_t packed[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int j = v * 8 + e * 2;
                float f0 = __uint_as_float(r[j]);
                float f1 = __uint_as_float(r[j + 1]);
                if (bias) {
                  f0 += __bfloat162float(bias[col0 + j]);
                  f1 += __bfloat162float(bias[col0 + j + 1]);
                }
                const bf162 h = __floats2bfloat162_rn(f0, f1);
                packed[e] = *reinterpret_cast<const uint32_t*>(&h);
              }
              reinterpret_cast<uint4*>(dst)[v] =
                  make_uint4(packed[0], packed[1], packed[2], packed[3]);
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              if (col0 + j < n) {
                float f = __uint_as_float(r[j]);
                if (bias) f += __bfloat162float(bias[col0 + j]);
                dst[j] = __float2bfloat16_rn(f);
              }
            }
          }
        }
      }
      tc_fence_before();
      // The four epilogue warps meet first, so one arrival per CTA (a remote
      // one from the peer) releases the accumulator.
      asm volatile("bar.sync 3, 128;" ::: "memory");
      if (threadIdx.x == 4 * 32) {
        if (leader) {
          mbar_arrive(bar_acc_empty + 8 * buf);
        } else {
          mbar_arrive_remote(acc_empty_leader + 8 * buf);
        }
      }
      // Peer copies of this CTA's 128 x 256 half tile, pushed after the
      // accumulator is released (the MMAs of the next tile run meanwhile):
      // warp q re-reads the 32 rows it just stored and sends each row as one
      // 512-byte segment (16 bytes per lane) to every peer, so the NVLink
      // writes are whole, contiguous lines rather than one 16-byte piece per
      // row per lane.
      if (peers.n > 0 && acc_ok) {
        const int col0 = nb * C::kBN;
        const int rbase = mb * 256 + int(rank) * 128 + q * 32;
        if (vec_ok && col0 + C::kBN <= n) {
          static_assert(C::kBN * 2 == 32 * 16, "one 16-byte piece per lane per row");
#pragma unroll 4
          for (int rr = 0; rr < 32; ++rr) {
            const int row = rbase + rr;
            if (row >= m) break;
            uint4* src = reinterpret_cast<uint4*>(out + size_t(row) * ldc + col0) + lane;
            const uint4 v = *src;
            for (int pi = 0; pi < peers.n; ++pi) {
              *reinterpret_cast<uint4*>(reinterpret_cast<char*>(src) + peers.delta[pi]) = v;
            }
          }
        } else {
          for (int rr = 0; rr < 32; ++rr) {
            const int row = rbase + rr;
            if (row >= m) break;
            for (int c = lane; c < C::kBN && col0 + c < n; c += 32) {
              bf16* src = out + size_t(row) * ldc + col0 + c;
              const bf16 v = *src;
              for (int pi = 0; pi < peers.n; ++pi) {
                *reinterpret_cast<bf16*>(reinterpret_cast<char*>(src) + peers.delta[pi]) = v;
              }
            }
          }
        }
      }
    }
    if (peers.n > 0) __threadfence_system();
  } else if (warp >= 8) {
    // ---------------------------------------------------------- dequantiser
    if constexpr (kW8) {
      const int dt = threadIdx.x - 8 * 32;
      constexpr int kItems = C::kHalf * 4;
      constexpr int kPerThread = kItems / (C::kDqWarps * 32);
      const uint32_t dq_leader = map_to_rank(bar_dq, 0);
      const uint16_t* sbits = reinterpret_cast<const uint16_t*>(scales);
      constexpr int kAhead = 4;
      auto load_scales = [&](int tile, int kb, uint32_t* dst) {
        const int nb = tile / num_m;
#pragma unroll
        for (int p = 0; p < kPerThread; ++p) {
          const int item = dt + p * (C::kDqWarps * 32);
          const int row = nb * C::kBN + int(rank) * C::kHalf + (item >> 2);
          const uint32_t v =
              (tile < num_tiles && row < n) ? sbits[size_t(row) * groups + kb] : 0u;
          dst[p] = v | (v << 16);
        }
      };
      int pf_tile = cluster, pf_kb = 0;
      uint32_t sq[kAhead][kPerThread];
#pragma unroll
      for (int d = 0; d < kAhead; ++d) {
        load_scales(pf_tile, pf_kb, sq[d]);
        if (++pf_kb == num_kb) {
          pf_kb = 0;
          pf_tile += num_clusters;
        }
      }
      const bf162 neg0 = __halves2bfloat162(__ushort_as_bfloat16(0x8000),
                                            __ushort_as_bfloat16(0x8000));
      int stage = 0;
      uint32_t phase = 0;
      int dstage = 0;
      uint32_t dphase = 0;
      int tile = cluster, kb = 0;
      while (true) {
#pragma unroll
        for (int d = 0; d < kAhead; ++d) {
          if (tile >= num_tiles) goto dequant2_done;
          // As in the epilogue, a failed wait skips the work but keeps the
          // thread in step with the named barrier below.
          const bool ok = mbar_wait(bar_fullq + 8 * stage, phase, abort_flag,
                                    B200_DEVICE_TIMEOUT_PIPELINE) &&
                          mbar_wait_cl(bar_dq_empty + 8 * dstage, dphase ^ 1, abort_flag,
                                       B200_DEVICE_TIMEOUT_PIPELINE);
          unsigned char* st = smem + stage * C::kStageBytes;
          unsigned char* bt = dq_ring + dstage * C::kDqBytes;
          const unsigned char* qt = st + C::kABytes;
#pragma unroll
          for (int p = 0; p < kPerThread; ++p) {
            if (!ok) break;
            const int item = dt + p * (C::kDqWarps * 32);
            const int r = item >> 2;
            const int j = item & 3;
            const uint4 raw = *reinterpret_cast<const uint4*>(qt + r * kBK + j * 16);
            const uint32_t s2bits = sq[d][p];
            const bf162 s2 = *reinterpret_cast<const bf162*>(&s2bits);
            uint32_t outw[8];
            const uint32_t words[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
            for (int wi = 0; wi < 4; ++wi) {
              const uint32_t b = words[wi] ^ 0x80808080u;
              const uint32_t f0 = __float_as_uint(s8_to_f32_biased<0>(b));
              const uint32_t f1 = __float_as_uint(s8_to_f32_biased<1>(b));
              const uint32_t f2 = __float_as_uint(s8_to_f32_biased<2>(b));
              const uint32_t f3 = __float_as_uint(s8_to_f32_biased<3>(b));
              uint32_t q01 = __byte_perm(f0, f1, 0x7632);
              uint32_t q23 = __byte_perm(f2, f3, 0x7632);
              bf162 d01 = __hfma2(*reinterpret_cast<bf162*>(&q01), s2, neg0);
              bf162 d23 = __hfma2(*reinterpret_cast<bf162*>(&q23), s2, neg0);
              outw[2 * wi] = *reinterpret_cast<uint32_t*>(&d01);
              outw[2 * wi + 1] = *reinterpret_cast<uint32_t*>(&d23);
            }
            unsigned char* rowp = bt + (r >> 3) * 1024 + (r & 7) * 128;
            const int c0 = (2 * j) ^ (r & 7);
            const int c1 = (2 * j + 1) ^ (r & 7);
            *reinterpret_cast<uint4*>(rowp + c0 * 16) =
                make_uint4(outw[0], outw[1], outw[2], outw[3]);
            *reinterpret_cast<uint4*>(rowp + c1 * 16) =
                make_uint4(outw[4], outw[5], outw[6], outw[7]);
          }
          fence_proxy_async_smem();
          // All dequant threads of this CTA meet, then one arrival per CTA.
          asm volatile("bar.sync 2, %0;" ::"r"(C::kDqWarps * 32) : "memory");
          if (dt == 0) {
            if (leader) {
              mbar_arrive(bar_dq + 8 * dstage);
            } else {
              mbar_arrive_remote(dq_leader + 8 * dstage);
            }
          }
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
          if (++dstage == C::kDqStages) {
            dstage = 0;
            dphase ^= 1;
          }
          load_scales(pf_tile, pf_kb, sq[d]);
          if (++pf_kb == num_kb) {
            pf_kb = 0;
            pf_tile += num_clusters;
          }
          if (++kb == num_kb) {
            kb = 0;
            tile += num_clusters;
          }
        }
      }
    dequant2_done:;
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(C::kTmemCols)
                 : "memory");
  }
}

// ------------------------------------------------------------------- host
PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault,
                                &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
  });
  return fn;
}

bool make_tmap(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
               int elem_bytes, int inner, int outer, int box_inner,
               int box_outer, CUtensorMapSwizzle swizzle) {
  auto fn = get_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {cuuint64_t(inner), cuuint64_t(outer)};
  cuuint64_t strides[1] = {cuuint64_t(inner) * elem_bytes};
  cuuint32_t box[2] = {cuuint32_t(box_inner), cuuint32_t(box_outer)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Host-side launch costs of a GEMM call, paid once instead of per call: a
// cache of encoded tensor maps (a map holds only the address, shape, box and
// swizzle it was encoded with, so equal keys give equal maps), and the
// dynamic shared-memory attribute set once per kernel and device.
struct TmapKey {
  const void* base;
  int dev, dtype, elem_bytes, inner, outer, box_inner, box_outer, swizzle;
  bool operator==(const TmapKey& o) const {
    return base == o.base && dev == o.dev && dtype == o.dtype && elem_bytes == o.elem_bytes &&
           inner == o.inner && outer == o.outer && box_inner == o.box_inner &&
           box_outer == o.box_outer && swizzle == o.swizzle;
  }
};
struct TmapEntry {
  TmapKey key;
  CUtensorMap map;
  bool valid = false;
};
constexpr int kTmapCacheSize = 128;
std::mutex g_tmap_mutex;
TmapEntry g_tmap_cache[kTmapCacheSize];
unsigned g_tmap_next = 0;

bool make_tmap_cached(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                      int elem_bytes, int inner, int outer, int box_inner, int box_outer,
                      CUtensorMapSwizzle swizzle) {
  int dev = 0;
  cudaGetDevice(&dev);
  const TmapKey key{base, dev, int(dtype), elem_bytes, inner, outer, box_inner, box_outer,
                    int(swizzle)};
  {
    std::lock_guard<std::mutex> lock(g_tmap_mutex);
    for (const TmapEntry& e : g_tmap_cache) {
      if (e.valid && e.key == key) {
        *map = e.map;
        return true;
      }
    }
  }
  if (!make_tmap(map, base, dtype, elem_bytes, inner, outer, box_inner, box_outer, swizzle)) {
    return false;
  }
  std::lock_guard<std::mutex> lock(g_tmap_mutex);
  TmapEntry& slot = g_tmap_cache[g_tmap_next++ % kTmapCacheSize];
  slot.key = key;
  slot.map = *map;
  slot.valid = true;
  return true;
}

template <auto kKernel>
cudaError_t ensure_smem_attr(int bytes) {
  static std::atomic<unsigned long long> done{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = dev >= 0 && dev < 64 ? 1ull << dev : 0ull;
  if (bit != 0 && (done.load(std::memory_order_acquire) & bit) != 0) return cudaSuccess;
  const cudaError_t e =
      cudaFuncSetAttribute(kKernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_release);
  return e;
}

int sm_count() {
  int dev = 0;
  cudaGetDevice(&dev);
  int count = 148;
  cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev);
  return count;
}

template <bool kW8, int kMSub, int kBN>
cudaError_t launch_cfg(const void* weight, const bf16* scales, const bf16* bias,
                       const bf16* input, bf16* output, int m, int n, int k,
                       int ldc, const PeerOuts& peers, cudaStream_t stream,
                       int splits = 1, float* partial = nullptr) {
  using C = Cfg<kW8, kMSub, kBN>;
  CUtensorMap tx, tw;
  // A short prompt (m < 128, one 128-row sub-tile) loads only its rows.
  const int a_rows = (kMSub == 1 && m < 128) ? (m + 7) / 8 * 8 : 128;
  if (!make_tmap_cached(&tx, input, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, k, m, kBK, a_rows,
                 CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  if (kW8) {
    if (!make_tmap_cached(&tw, weight, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, k, n, kBK, kBN,
                   CU_TENSOR_MAP_SWIZZLE_NONE))
      return cudaErrorInvalidValue;
  } else {
    if (!make_tmap_cached(&tw, weight, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, k, n, kBK,
                   kBN, CU_TENSOR_MAP_SWIZZLE_128B))
      return cudaErrorInvalidValue;
  }
  auto kernel = gemm_tc_kernel<kW8, kMSub, kBN>;
  cudaError_t e = ensure_smem_attr<gemm_tc_kernel<kW8, kMSub, kBN>>(C::kSmemBytes);
  if (e != cudaSuccess) return e;
  const int tiles = ((m + C::kBM - 1) / C::kBM) * ((n + kBN - 1) / kBN);
  // K split over grid z: chunks of whole 64-wide k-blocks
  const int kchunk = splits > 1 ? ((k + splits - 1) / splits + kBK - 1) / kBK * kBK : k;
  const int zs = (k + kchunk - 1) / kchunk;
  const int per_z = sm_count() / zs > 0 ? sm_count() / zs : 1;
  const int grid = tiles < per_z ? tiles : per_z;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, zs);
  cfg.blockDim = dim3(C::kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, tx, tw, scales, bias, output, m, n, k, ldc, peers,
                            a_rows, kchunk, splits > 1 ? partial : nullptr);
}

template <bool kW8>
cudaError_t launch_pair(const void* weight, const bf16* scales, const bf16* bias,
                        const bf16* input, bf16* output, int m, int n, int k,
                        int ldc, const PeerOuts& peers, cudaStream_t stream) {
  using C = Cfg2<kW8>;
  CUtensorMap tx, tw;
  if (!make_tmap_cached(&tx, input, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, k, m, kBK, 128,
                 CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  if (kW8) {
    if (!make_tmap_cached(&tw, weight, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, k, n, kBK, C::kHalf,
                   CU_TENSOR_MAP_SWIZZLE_NONE))
      return cudaErrorInvalidValue;
  } else {
    if (!make_tmap_cached(&tw, weight, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, k, n, kBK, C::kHalf,
                   CU_TENSOR_MAP_SWIZZLE_128B))
      return cudaErrorInvalidValue;
  }
  auto kernel = gemm_tc2_kernel<kW8>;
  cudaError_t e = ensure_smem_attr<gemm_tc2_kernel<kW8>>(C::kSmemBytes);
  if (e != cudaSuccess) return e;
  const int tiles = ((m + 255) / 256) * ((n + C::kBN - 1) / C::kBN);
  const int pairs = sm_count() / 2;
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
  return cudaLaunchKernelEx(&cfg, kernel, tx, tw, scales, bias, output, m, n, k, ldc, peers);
}

bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}


// Tile-shape choice: the largest tile that still gives every SM work.
// B200_GEMM_TILE=pair|256x128|128x256|128x128|128x64 overrides it (tuning only).
enum class Tile { kPair256x256, k256x128, k128x256, k128x128, k128x64, k128x32 };

// BF16 prefers the CTA-pair 256x256 tile, then 128x256 (one N=256 MMA per
// k-step reads less shared memory per FLOP than two M=128 x N=128 MMAs);
// INT8 weights prefer 256x128, which dequantises each weight tile once for
// 256 token rows (the pair kernel's INT8 form measured slower: the
// dequant-to-MMA hand-off across the two SMs limits it).
Tile choose_tile(bool w8, int m, int n) {
  static const char* forced = getenv("B200_GEMM_TILE");
  if (forced) {
    if (!strcmp(forced, "pair")) return Tile::kPair256x256;
    if (!strcmp(forced, "256x128")) return Tile::k256x128;
    if (!strcmp(forced, "128x256")) return Tile::k128x256;
    if (!strcmp(forced, "128x128")) return Tile::k128x128;
    if (!strcmp(forced, "128x64")) return Tile::k128x64;
    if (!strcmp(forced, "128x32") && !w8) return Tile::k128x32;
  }
  const long long sms = sm_count();
  const long long t256x128 = ((m + 255) / 256) * (long long)((n + 127) / 128);
  const long long t128x128 = ((m + 127) / 128) * (long long)((n + 127) / 128);
  const long long t128x256 = ((m + 127) / 128) * (long long)((n + 255) / 256);
  const long long tpair = ((m + 255) / 256) * (long long)((n + 255) / 256);
  if (!w8 && tpair >= sms / 2) return Tile::kPair256x256;
  if (!w8 && t128x256 >= sms) return Tile::k128x256;
  if (t256x128 >= sms) return Tile::k256x128;
  if (t128x128 >= sms / 2) return Tile::k128x128;
  // Few tokens and few columns: each tile walks all of K, so the GEMM takes
  // as long as one tile's K walk; narrower BF16 tiles put more SMs on it
  // (same per-element K order, so the same results).
  const long long t128x64 = ((m + 127) / 128) * (long long)((n + 63) / 64);
  if (!w8 && t128x64 < sms / 4) return Tile::k128x32;
  return Tile::k128x64;
}

template <bool kW8>
cudaError_t launch_tile(Tile t, const void* weight, const bf16* scales,
                        const bf16* bias, const bf16* input, bf16* output,
                        int m, int n, int k, int ldc, const PeerOuts& peers,
                        cudaStream_t stream) {
  switch (t) {
    case Tile::kPair256x256:
      return launch_pair<kW8>(weight, scales, bias, input, output, m, n, k, ldc, peers, stream);
    case Tile::k256x128:
      return launch_cfg<kW8, 2, 128>(weight, scales, bias, input, output, m, n, k, ldc, peers,
                                     stream);
    case Tile::k128x256:
      return launch_cfg<kW8, 1, 256>(weight, scales, bias, input, output, m, n, k, ldc, peers,
                                     stream);
    case Tile::k128x128:
      return launch_cfg<kW8, 1, 128>(weight, scales, bias, input, output, m, n, k, ldc, peers,
                                     stream);
    case Tile::k128x32:
      if constexpr (!kW8) {
        return launch_cfg<false, 1, 32>(weight, scales, bias, input, output, m, n, k, ldc, peers,
                                        stream);
      }
      [[fallthrough]];
    default:
      return launch_cfg<kW8, 1, 64>(weight, scales, bias, input, output, m, n, k, ldc, peers,
                                    stream);
  }
}

}  // namespace

bool encode_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                    int elem_bytes, int inner, int outer, int box_inner, int box_outer,
                    CUtensorMapSwizzle swizzle) {
  return make_tmap_cached(map, base, dtype, elem_bytes, inner, outer, box_inner, box_outer,
                          swizzle);
}

bool gemm_tc_supported(bool w8, const void* weight, const void* input,
                       const void* output, int m, int n, int k) {
  (void)output;
  if (m <= 0 || n <= 0 || k <= 0) return false;
  if (k % (w8 ? 16 : 8) != 0) return false;  // TMA row stride: 16-byte multiple
  if (!aligned16(weight) || !aligned16(input)) return false;
  return get_encode_fn() != nullptr;
}

// ---------------------------------------------------------------------------
// Two-pass W8A16 prefill for many tokens: the INT8 weights are dequantised
// once into BF16 -- bf16(q * s), the exact value the in-kernel dequant feeds
// the MMA -- and the CTA-pair BF16 GEMM runs on them.  At M >= 1024 the extra
// pass over W (1 byte read + 2 written per weight) costs a few percent of
// the GEMM, while the in-kernel hand-off of dequantised tiles to the tensor
// cores limits the one-pass kernel to about half the BF16 rate.  The BF16
// weights go to a device buffer owned by the library (one per device,
// kScratchCap bytes at most; W is processed in row blocks that fit).  The
// buffer exists only after an explicit b200_gemm_reserve_scratch on that
// device (a GEMM call never allocates); without it the one-pass kernels run
// (same results).
namespace {

constexpr size_t kScratchCap = size_t(256) << 20;
constexpr int kTwoPassMinTokens = 1024;
// Measured: the extra pass over W pays off only for large outputs (e.g.
// 8192 x 4864 or 2048 x 151936); below, the one-pass kernels are faster.
constexpr double kTwoPassMinOutputs = 32.0 * 1024 * 1024;

struct Scratch {
  void* ptr = nullptr;
  size_t bytes = 0;
};
std::mutex g_scratch_mutex;
Scratch g_scratch[64];

cudaError_t scratch_get(size_t want, bool may_allocate, Scratch* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  Scratch& sc = g_scratch[dev];
  if (sc.ptr == nullptr && may_allocate) {
    const size_t bytes = want < kScratchCap ? want : kScratchCap;
    e = cudaMalloc(&sc.ptr, bytes);
    if (e != cudaSuccess) {
      sc.ptr = nullptr;
      cudaGetLastError();
      return e;
    }
    sc.bytes = bytes;
  }
  *out = sc;
  return sc.ptr != nullptr ? cudaSuccess : cudaErrorMemoryAllocation;
}

// rows x k INT8 + BF16 group-64 scales -> rows x k BF16, 16 weights per thread.
__global__ void __launch_bounds__(256)
dequant_w8_kernel(const int8_t* __restrict__ q, const uint16_t* __restrict__ scales,
                  int groups, bf16* __restrict__ out, int rows, int k) {
  const int cpr = k >> 4;  // 16-byte chunks per row
  const size_t total = size_t(rows) * cpr;
  const bf162 neg0 = __halves2bfloat162(__ushort_as_bfloat16(0x8000),
                                        __ushort_as_bfloat16(0x8000));
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < total;
       i += size_t(gridDim.x) * blockDim.x) {
    const size_t row = i / cpr;
    const int c = int(i - row * cpr);
    const uint4 raw = reinterpret_cast<const uint4*>(q)[i];
    const uint32_t sv = scales[row * groups + (c >> 2)];
    const uint32_t s2bits = sv | (sv << 16);
    const bf162 s2 = *reinterpret_cast<const bf162*>(&s2bits);
    uint32_t w[8];
    const uint32_t words[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int wi = 0; wi < 4; ++wi) {
      const uint32_t b = words[wi] ^ 0x80808080u;
      const uint32_t f0 = __float_as_uint(s8_to_f32_biased<0>(b));
      const uint32_t f1 = __float_as_uint(s8_to_f32_biased<1>(b));
      const uint32_t f2 = __float_as_uint(s8_to_f32_biased<2>(b));
      const uint32_t f3 = __float_as_uint(s8_to_f32_biased<3>(b));
      uint32_t q01 = __byte_perm(f0, f1, 0x7632);
      uint32_t q23 = __byte_perm(f2, f3, 0x7632);
      bf162 d01 = __hfma2(*reinterpret_cast<bf162*>(&q01), s2, neg0);
      bf162 d23 = __hfma2(*reinterpret_cast<bf162*>(&q23), s2, neg0);
      w[2 * wi] = *reinterpret_cast<uint32_t*>(&d01);
      w[2 * wi + 1] = *reinterpret_cast<uint32_t*>(&d23);
    }
    uint4* dst = reinterpret_cast<uint4*>(out) + 2 * i;
    dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
    dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
  }
}

cudaError_t gemm_w8_two_pass(const void* weight, const bf16* scales, const bf16* bias,
                             const bf16* input, bf16* output, int m, int n, int k, int ldc,
                             const PeerOuts& peers, const Scratch& sc, cudaStream_t stream) {
  const size_t row_bytes = size_t(k) * 2;
  int block = int(sc.bytes / row_bytes) / 256 * 256;
  if (block <= 0) return cudaErrorMemoryAllocation;
  if (block > n) block = n;
  const int groups = (k + 63) / 64;
  const int8_t* q = static_cast<const int8_t*>(weight);
  const uint16_t* sb = reinterpret_cast<const uint16_t*>(scales);
  bf16* wb = static_cast<bf16*>(sc.ptr);
  for (int n0 = 0; n0 < n; n0 += block) {
    const int nr = n - n0 < block ? n - n0 : block;
    const size_t chunks = size_t(nr) * (k / 16);
    int grid = int((chunks + 255) / 256);
    if (grid > 148 * 8) grid = 148 * 8;
    dequant_w8_kernel<<<grid, 256, 0, stream>>>(q + size_t(n0) * k, sb + size_t(n0) * groups,
                                                groups, wb, nr, k);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    e = launch_tile<false>(choose_tile(false, m, nr), wb, nullptr, bias ? bias + n0 : nullptr,
                           input, output + n0, m, nr, k, ldc, peers, stream);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

// Sum of the K-split partials in split order, + bias, BF16 RNE.
__global__ void __launch_bounds__(256)
splitk_reduce_kernel(const float* __restrict__ partial, int splits, const bf16* __restrict__ bias,
                     bf16* __restrict__ out, int m, int n, int ldc) {
  pdl_launch_dependents();
  pdl_wait_primary();
  const size_t total = size_t(m) * n;
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < total;
       i += size_t(gridDim.x) * blockDim.x) {
    const int row = int(i / n), col = int(i - size_t(row) * n);
    float acc = partial[i];
    for (int z = 1; z < splits; ++z) acc += partial[size_t(z) * total + i];
    if (bias) acc += __bfloat162float(bias[col]);
    out[size_t(row) * ldc + col] = __float2bfloat16_rn(acc);
  }
}

// Short prompts in the fast summation order: the few output tiles each walk
// K split over grid z (FP32 partials into the reserved buffer, reduced in a
// fixed order).  Returns cudaErrorNotSupported when it does not apply.
// Measured on B200: with K = 4864 the split halves a 32-token GEMM (32 ->
// 16 us); with K = 896 the partial traffic and the extra launch cost more
// than the split gains (e.g. 128 x 896 -> 896: 10.5 -> 22.9 us), so only
// long K splits.
constexpr int kSplitMaxTokens = 128;
constexpr int kSplitMinK = 2048;
cudaError_t gemm_split_k(bool w8, const void* weight, const bf16* scales, const bf16* bias,
                         const bf16* input, bf16* output, int m, int n, int k, int ldc,
                         cudaStream_t stream) {
  if (m > kSplitMaxTokens || k < kSplitMinK || summation_order() != B200_ORDER_FAST ||
      getenv("B200_GEMM_NO_SPLITK") != nullptr) {
    return cudaErrorNotSupported;
  }
  const int bn = w8 ? 64 : 32;
  const int tiles = (n + bn - 1) / bn;  // one 128-row tile covers the prompt
  const int num_kb = (k + kBK - 1) / kBK;
  int splits = sm_count() / tiles;
  if (splits > num_kb) splits = num_kb;
  if (splits > 16) splits = 16;
  if (splits < 2) return cudaErrorNotSupported;
  const int kchunk = ((k + splits - 1) / splits + kBK - 1) / kBK * kBK;
  const int zs = (k + kchunk - 1) / kchunk;
  Scratch sc;
  if (scratch_get(kScratchCap, false, &sc) != cudaSuccess ||
      sc.bytes < size_t(zs) * m * n * sizeof(float)) {
    return cudaErrorNotSupported;
  }
  float* part = static_cast<float*>(sc.ptr);
  cudaError_t e = w8 ? launch_cfg<true, 1, 64>(weight, scales, nullptr, input, output, m, n, k,
                                               ldc, PeerOuts{}, stream, splits, part)
                     : launch_cfg<false, 1, 32>(weight, scales, nullptr, input, output, m, n, k,
                                                ldc, PeerOuts{}, stream, splits, part);
  if (e != cudaSuccess) return e;
  const size_t total = size_t(m) * n;
  int grid = int((total + 255) / 256);
  if (grid > 4 * sm_count()) grid = 4 * sm_count();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, splitk_reduce_kernel, (const float*)part, zs, bias, output, m,
                            n, ldc);
}

}  // namespace

// B200_GEMM_W8T=1 selects the TMEM-weight W8A16 kernel for every prompt
// length (tuning / tests).
bool use_w8t() {
  static const bool on = [] {
    const char* e = getenv("B200_GEMM_W8T");
    return e != nullptr && strcmp(e, "1") == 0;
  }();
  return on;
}

cudaError_t reserve_gemm_scratch(size_t bytes) {
  Scratch sc;
  return scratch_get(bytes == 0 ? kScratchCap : bytes, true, &sc);
}

// Prompts of < 1024 tokens on the TMEM-weight kernel unless
// B200_GEMM_W8T_SHORT=0 (read at every call, for measurement).
// Cluster split-K for short prompts on narrow matrices unless
// B200_GEMM_CSPLIT=0 (read at every call).
static bool use_cluster_split() {
  const char* e = getenv("B200_GEMM_CSPLIT");
  return e == nullptr || strcmp(e, "0") != 0;
}

static bool use_w16t(int m, int n, int k) {
  const char* e = getenv("B200_GEMM_W16T");
  if (e != nullptr) return strcmp(e, "1") == 0;
  return m <= 32 || n >= 16384 || k >= 2048;
}

static bool use_w8t_short() {
  const char* e = getenv("B200_GEMM_W8T_SHORT");
  return e == nullptr || strcmp(e, "0") != 0;
}

cudaError_t launch_gemm_tc_peers(bool w8, const void* weight, const bf16* scales,
                                 const bf16* bias, const bf16* input, bf16* output,
                                 int m, int n, int k, int ldc, const PeerOuts& peers,
                                 cudaStream_t stream) {
  if (peers.n == 0 && m <= 512 && summation_order() == B200_ORDER_FAST &&
      use_cluster_split() && gemm_w8t_supported(weight, input, output, m, n, k)) {
    const cudaError_t e = launch_gemm_cluster_split(w8, weight, scales, bias, input, output,
                                                    m, n, k, ldc, stream);
    if (e != cudaErrorNotSupported) return e;
  }
  if (peers.n == 0 && m <= kSplitMaxTokens) {
    const cudaError_t e =
        gemm_split_k(w8, weight, scales, bias, input, output, m, n, k, ldc, stream);
    if (e != cudaErrorNotSupported) return e;
  }
  if (w8 && m >= kTwoPassMinTokens && double(m) * double(n) >= kTwoPassMinOutputs &&
      !getenv("B200_GEMM_ONE_PASS")) {
    // Only a buffer reserved beforehand (b200_gemm_reserve_scratch) is used;
    // one too small for a 256-row block of this K leaves the one-pass path.
    Scratch sc;
    if (scratch_get(kScratchCap, false, &sc) == cudaSuccess &&
        sc.bytes / (size_t(k) * 2) >= 256) {
      return gemm_w8_two_pass(weight, scales, bias, input, output, m, n, k, ldc, peers, sc,
                              stream);
    }
  }
  // One pass with the dequantised weights in TMEM (gemm_w8t.cu) at every
  // prompt length (short prompts get a token tile fitted to them: the
  // weights stay the MMA's M side, no token padding to 128; measured faster
  // than the shared-memory dequant kernel at 32, 128 and 512 tokens, 2x on
  // 896 -> 151936); its epilogue has no peer stores, so the sharded form
  // keeps the shared-memory dequant kernels.
  // Narrow matrices (<= 1024 outputs) at 129..2048 tokens stay on the
  // shared-memory dequant kernel, measured faster there (few weight tiles:
  // the tokens-as-M tiling spreads them over more SMs).
  // B200_GEMM_W8T_NARROW=1 sends them to the TMEM-weight kernel.
  const char* nv = getenv("B200_GEMM_W8T_NARROW");
  const bool narrow = m > 128 && m <= 2048 && n <= 1024 && !(nv != nullptr && nv[0] == '1');
  if (w8 && peers.n == 0 && !narrow &&
      (m >= kTwoPassMinTokens || use_w8t_short() || use_w8t()) &&
      gemm_w8t_supported(weight, input, output, m, n, k)) {
    return launch_gemm_w8t(weight, scales, bias, input, output, m, n, k, ldc, stream);
  }
  // BF16, <= 128 tokens: the transposed form (weights the MMA's M side,
  // token tile fitted to the prompt) where it measured faster: <= 32 tokens
  // (e.g. 32 x 896 -> 151936: 60.7 -> 47.6 us), and up to 128 tokens for
  // wide or long-K matrices (128 x 896 -> 4864 stays on the default kernel:
  // 7.3 vs 8.6 us).  B200_GEMM_W16T=1 / 0 forces it on / off.
  if (!w8 && peers.n == 0 && m <= 128 && use_w16t(m, n, k) &&
      gemm_w8t_supported(weight, input, output, m, n, k)) {
    return launch_gemm_w16t(static_cast<const bf16*>(weight), bias, input, output, m, n, k,
                            ldc, stream);
  }
  const Tile t = choose_tile(w8, m, n);
  return w8 ? launch_tile<true>(t, weight, scales, bias, input, output, m, n, k, ldc, peers,
                                stream)
            : launch_tile<false>(t, weight, scales, bias, input, output, m, n, k, ldc, peers,
                                 stream);
}

cudaError_t launch_gemm_tc(bool w8, const void* weight, const bf16* scales,
                           const bf16* bias, const bf16* input, bf16* output,
                           int m, int n, int k, cudaStream_t stream) {
  return launch_gemm_tc_peers(w8, weight, scales, bias, input, output, m, n, k, n, PeerOuts{},
                              stream);
}

}  // namespace b200
