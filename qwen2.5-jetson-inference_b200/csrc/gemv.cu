// Decode GEMV (M = 1) and fused LM-head GEMV + argmax for sm_100a.
//
// Replaces the reference's gemv_bf16 / gemv_w8a16 / lm_head_bf16 /
// argmax_bf16 (reference src/cuda/kernels.cu:326-603, 953-1041, 1540-1655).
//
// Design (B200): the GEMV is a pure HBM stream of the weight matrix, so the
// kernel is organised around bytes in flight rather than around rows:
//  * a "team" of TPR threads owns R consecutive rows; each thread walks the
//    row in 16-byte chunks (c = t, t+TPR, ...), loading the same chunk of all
//    R rows, so one shared-memory read of x feeds R rows;
//  * U chunk-columns are loaded before any arithmetic (R*U 128-bit loads in
//    flight per thread, non-allocating in L1);
//  * INT8 -> FP32 uses the exact magic-number conversion (two ALU ops per
//    byte, no I2F), the 16 products of a chunk are summed in FP32 and the
//    chunk sum is multiplied by the BF16 group scale once (a chunk never
//    straddles a 64-wide group);
//  * TPR / R are picked per shape so that small matrices spread over every
//    SM and large ones keep each thread busy (choose_config);
//  * launches carry the programmatic-dependent-launch attribute: the weight
//    prefetch is issued before griddepcontrol.wait, so a chain of Linear
//    calls overlaps one kernel's tail with the next one's weight stream.
//    Nothing is written to global memory before the wait.
//
// The LM-head form adds a per-CTA argmax over the BF16-rounded logits
// (lowest index on ties) written to the caller's workspace, and a one-CTA
// reduction kernel (launched with PDL) that writes the final index.

#include <atomic>
#include <cfloat>
#include <climits>
#include <cstdlib>
#include <cstdio>
#include <cstring>

#include "b200_linear.h"
#include "common.cuh"
#include "gemv_math.cuh"
#include "kernels.h"

namespace b200 {

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 v;
  asm volatile(
      "ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p));
  return v;
}

// acc += sum_{j<4} q_j * x_j for the four int8 of one packed word.
__device__ __forceinline__ float dot4_s8(uint32_t packed, const float* x,
                                         float acc) {
  const uint32_t b = packed ^ 0x80808080u;
  acc = fmaf(s8_to_f32_biased<0>(b), x[0], acc);
  acc = fmaf(s8_to_f32_biased<1>(b), x[1], acc);
  acc = fmaf(s8_to_f32_biased<2>(b), x[2], acc);
  acc = fmaf(s8_to_f32_biased<3>(b), x[3], acc);
  return acc;
}

__device__ __forceinline__ float dot2_bf16(uint32_t w, float x0, float x1,
                                           float acc) {
  acc = fmaf(bf16_lo(w), x0, acc);
  acc = fmaf(bf16_hi(w), x1, acc);
  return acc;
}

template <bool kW8, int kTPR, int kR>
__global__ void __launch_bounds__(kThreads, 2)
gemv_stream_kernel(const void* __restrict__ weight,
                   const bf16* __restrict__ scales,
                   const bf16* __restrict__ bias,
                   const bf16* __restrict__ input, bf16* __restrict__ output,
                   int n_rows, int k, float* __restrict__ block_value,
                   int* __restrict__ block_index) {
  constexpr int kTeams = kThreads / kTPR;
  constexpr int kU = kR == 1 ? 4 : 2;  // chunk columns in flight per thread
  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint32_t* xs = reinterpret_cast<uint32_t*>(smem_raw);  // k bf16 (pairs)
  __shared__ float red_val[kThreads / 32 > 0 ? kThreads / 32 : 1][kR];
  __shared__ float team_best[kTeams];
  __shared__ int team_best_index[kTeams];

  const int team = threadIdx.x / kTPR;
  const int t = threadIdx.x % kTPR;
  const int row0 = (blockIdx.x * kTeams + team) * kR;
  const int chunks = kW8 ? (k >> 4) : (k >> 3);
  const int groups = (k + 63) >> 6;
  const size_t row_bytes = kW8 ? size_t(k) : size_t(k) * 2;
  const unsigned char* wbase = static_cast<const unsigned char*>(weight);

  bool valid[kR];
  const unsigned char* wrow[kR];
#pragma unroll
  for (int r = 0; r < kR; ++r) {
    valid[r] = row0 + r < n_rows;
    wrow[r] = wbase + size_t(valid[r] ? row0 + r : 0) * row_bytes;
  }

  // First batch of weight loads does not depend on the previous kernel.
  uint4 w[kU][kR];
  int base = t;
#pragma unroll
  for (int u = 0; u < kU; ++u) {
    const int c = base + u * kTPR;
#pragma unroll
    for (int r = 0; r < kR; ++r) {
      w[u][r] = (c < chunks && valid[r]) ? ld_stream16(wrow[r] + size_t(c) * 16)
                                         : make_uint4(0, 0, 0, 0);
    }
  }
  pdl_launch_dependents();
  pdl_wait_primary();

  // Stage x (BF16) in shared memory with 16-byte copies.
  {
    const uint4* src = reinterpret_cast<const uint4*>(input);
    uint4* dst = reinterpret_cast<uint4*>(xs);
    for (int i = threadIdx.x; i < (k >> 3); i += kThreads) dst[i] = src[i];
  }
  __syncthreads();

  float acc[kR];
#pragma unroll
  for (int r = 0; r < kR; ++r) acc[r] = 0.0f;

  while (true) {
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int c = base + u * kTPR;
      if (c < chunks) {
        if constexpr (kW8) {
          const uint4 xa = reinterpret_cast<const uint4*>(xs)[2 * c];
          const uint4 xb = reinterpret_cast<const uint4*>(xs)[2 * c + 1];
          float xf[16];
          xf[0] = bf16_lo(xa.x); xf[1] = bf16_hi(xa.x);
          xf[2] = bf16_lo(xa.y); xf[3] = bf16_hi(xa.y);
          xf[4] = bf16_lo(xa.z); xf[5] = bf16_hi(xa.z);
          xf[6] = bf16_lo(xa.w); xf[7] = bf16_hi(xa.w);
          xf[8] = bf16_lo(xb.x); xf[9] = bf16_hi(xb.x);
          xf[10] = bf16_lo(xb.y); xf[11] = bf16_hi(xb.y);
          xf[12] = bf16_lo(xb.z); xf[13] = bf16_hi(xb.z);
          xf[14] = bf16_lo(xb.w); xf[15] = bf16_hi(xb.w);
#pragma unroll
          for (int r = 0; r < kR; ++r) {
            float p = 0.0f;
            p = dot4_s8(w[u][r].x, xf + 0, p);
            p = dot4_s8(w[u][r].y, xf + 4, p);
            p = dot4_s8(w[u][r].z, xf + 8, p);
            p = dot4_s8(w[u][r].w, xf + 12, p);
            const float s =
                valid[r] ? __bfloat162float(
                               scales[size_t(row0 + r) * groups + (c >> 2)])
                         : 0.0f;
            acc[r] = fmaf(p, s, acc[r]);
          }
        } else {
          const uint4 xa = reinterpret_cast<const uint4*>(xs)[c];
          const float x0 = bf16_lo(xa.x), x1 = bf16_hi(xa.x);
          const float x2 = bf16_lo(xa.y), x3 = bf16_hi(xa.y);
          const float x4 = bf16_lo(xa.z), x5 = bf16_hi(xa.z);
          const float x6 = bf16_lo(xa.w), x7 = bf16_hi(xa.w);
#pragma unroll
          for (int r = 0; r < kR; ++r) {
            float a = acc[r];
            a = dot2_bf16(w[u][r].x, x0, x1, a);
            a = dot2_bf16(w[u][r].y, x2, x3, a);
            a = dot2_bf16(w[u][r].z, x4, x5, a);
            a = dot2_bf16(w[u][r].w, x6, x7, a);
            acc[r] = a;
          }
        }
      }
    }
    base += kU * kTPR;
    if (base >= chunks) break;
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int c = base + u * kTPR;
#pragma unroll
      for (int r = 0; r < kR; ++r) {
        w[u][r] = (c < chunks && valid[r])
                      ? ld_stream16(wrow[r] + size_t(c) * 16)
                      : make_uint4(0, 0, 0, 0);
      }
    }
  }

  // Team reduction.
  constexpr int kWarpSpan = kTPR < 32 ? kTPR : 32;
#pragma unroll
  for (int r = 0; r < kR; ++r) {
#pragma unroll
    for (int off = kWarpSpan / 2; off > 0; off >>= 1) {
      acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], off);
    }
  }
  if constexpr (kTPR > 32) {
    constexpr int kWarpsPerTeam = kTPR / 32;
    const int warp = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) {
#pragma unroll
      for (int r = 0; r < kR; ++r) red_val[warp][r] = acc[r];
    }
    __syncthreads();
    if (t == 0) {
#pragma unroll
      for (int r = 0; r < kR; ++r) {
        float s = 0.0f;
#pragma unroll
        for (int i = 0; i < kWarpsPerTeam; ++i) s += red_val[warp + i][r];
        acc[r] = s;
      }
    }
  }

  if (t == 0) {
    float best = -FLT_MAX;
    int best_index = INT_MAX;
#pragma unroll
    for (int r = 0; r < kR; ++r) {
      if (valid[r]) {
        const float b = bias ? __bfloat162float(bias[row0 + r]) : 0.0f;
        const bf16 y = __float2bfloat16_rn(acc[r] + b);
        output[row0 + r] = y;
        argmax_update(best, best_index, __bfloat162float(y), row0 + r);
      }
    }
    if (block_value != nullptr) {
      team_best[team] = best;
      team_best_index[team] = best_index;
    }
  }
  if (block_value != nullptr) {
    __syncthreads();
    if (threadIdx.x == 0) {
      float best = -FLT_MAX;
      int best_index = INT_MAX;
      for (int i = 0; i < kTeams; ++i) {
        argmax_update(best, best_index, team_best[i], team_best_index[i]);
      }
      block_value[blockIdx.x] = best;
      block_index[blockIdx.x] = best_index;
    }
  }
}

// Any alignment / any K: one warp per row, scalar loads.  Also the LM-head
// form with 8 rows per CTA, so ceil(vocab/8) CTAs match the reference's
// workspace sizing (src/qwen2.cpp:193-198).
template <bool kW8>
__global__ void __launch_bounds__(kThreads)
gemv_generic_kernel(const void* __restrict__ weight,
                    const bf16* __restrict__ scales,
                    const bf16* __restrict__ bias,
                    const bf16* __restrict__ input, bf16* __restrict__ output,
                    int n_rows, int k, float* __restrict__ block_value,
                    int* __restrict__ block_index) {
  __shared__ float row_val[kThreads / 32];
  pdl_launch_dependents();
  pdl_wait_primary();
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (kThreads / 32) + warp;
  const int groups = (k + 63) >> 6;
  float acc = 0.0f;
  if (row < n_rows) {
    if constexpr (kW8) {
      const int8_t* w = static_cast<const int8_t*>(weight) + size_t(row) * k;
      const bf16* s = scales + size_t(row) * groups;
      for (int i = lane; i < k; i += 32) {
        acc = fmaf(float(w[i]) * __bfloat162float(s[i >> 6]),
                   __bfloat162float(input[i]), acc);
      }
    } else {
      const bf16* w = static_cast<const bf16*>(weight) + size_t(row) * k;
      for (int i = lane; i < k; i += 32) {
        acc = fmaf(__bfloat162float(w[i]), __bfloat162float(input[i]), acc);
      }
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    acc += __shfl_xor_sync(0xffffffffu, acc, off);
  }
  if (lane == 0) {
    float v = -FLT_MAX;
    if (row < n_rows) {
      const float b = bias ? __bfloat162float(bias[row]) : 0.0f;
      const bf16 y = __float2bfloat16_rn(acc + b);
      output[row] = y;
      v = __bfloat162float(y);
    }
    row_val[warp] = v;
  }
  if (block_value != nullptr) {
    __syncthreads();
    if (threadIdx.x == 0) {
      float best = -FLT_MAX;
      int best_index = INT_MAX;
      for (int i = 0; i < kThreads / 32; ++i) {
        const int r = blockIdx.x * (kThreads / 32) + i;
        if (r < n_rows) argmax_update(best, best_index, row_val[i], r);
      }
      block_value[blockIdx.x] = best;
      block_index[blockIdx.x] = best_index;
    }
  }
}

// Final argmax over per-CTA (value, index) pairs; one CTA.
__global__ void __launch_bounds__(1024)
argmax_partials_kernel(const float* __restrict__ block_value,
                       const int* __restrict__ block_index, int count,
                       int* __restrict__ argmax) {
  __shared__ float sv[32];
  __shared__ int si[32];
  pdl_wait_primary();
  float best = -FLT_MAX;
  int best_index = INT_MAX;
  for (int i = threadIdx.x; i < count; i += blockDim.x) {
    argmax_update(best, best_index, block_value[i], block_index[i]);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, off);
    const int oi = __shfl_xor_sync(0xffffffffu, best_index, off);
    argmax_update(best, best_index, ov, oi);
  }
  const int warp = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    sv[warp] = best;
    si[warp] = best_index;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = -FLT_MAX;
    int bi = INT_MAX;
    for (int i = 0; i < int(blockDim.x >> 5); ++i) argmax_update(b, bi, sv[i], si[i]);
    *argmax = bi == INT_MAX ? 0 : bi;
  }
}

// Argmax over BF16 values, one CTA (n is a vocabulary, not a matrix).
__global__ void __launch_bounds__(1024)
argmax_bf16_kernel(const bf16* __restrict__ values, int n,
                   int* __restrict__ out) {
  __shared__ float sv[32];
  __shared__ int si[32];
  pdl_wait_primary();
  float best = -FLT_MAX;
  int best_index = INT_MAX;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    argmax_update(best, best_index, __bfloat162float(values[i]), i);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, off);
    const int oi = __shfl_xor_sync(0xffffffffu, best_index, off);
    argmax_update(best, best_index, ov, oi);
  }
  const int warp = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    sv[warp] = best;
    si[warp] = best_index;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = -FLT_MAX;
    int bi = INT_MAX;
    for (int i = 0; i < int(blockDim.x >> 5); ++i) argmax_update(b, bi, sv[i], si[i]);
    *out = bi == INT_MAX ? 0 : bi;
  }
}


// ---------------------------------------------------------------------------
// Main decode path: weight tiles streamed by the TMA engine.
//
// One persistent CTA per SM.  Warp 0 (one lane) is the producer: for each
// tile of kTileRows consecutive rows -- a contiguous byte range of W, plus
// the matching contiguous range of the W8 scales -- it issues 1-D bulk
// copies (cp.async.bulk) into a ring of shared-memory stages guarded by
// full/empty mbarriers.  Because the weights never depend on the previous
// kernel, the producer starts before griddepcontrol.wait and the ring
// keeps ~100-200 KB per SM in flight regardless of how long the arithmetic
// takes.  Warps 1..8 are consumers: warp w owns kR rows of every tile; lane
// l handles 16-byte chunks c = l, l+32, ... of those rows, reading x from a
// shared FP32 copy laid out as kEPC/4 "planes" (plane p holds elements
// 4p..4p+3 of every chunk) so that consecutive lanes read consecutive
// 16-byte words (no bank conflicts).  The INT8 products use the sm_100
// packed FP32 instructions (2 elements per FADD2 / FFMA2).
// ---------------------------------------------------------------------------
// Reference summation order (opt-in, b200_set_summation_order).  The
// reference decode kernels (src/cuda/kernels.cu:359-384, 438-490, 492-568,
// 953-1041; built with --use_fast_math, so every FP32 add / mul / fma
// flushes denormals) sum a row as follows: lane l of the row's warp(s)
// walks chunks c = l + 32*ws, l + 32*ws + 32*W, ... (ws: the warp's slice of
// a row split over W warps); each chunk's dot product is a fresh chain
// (W8A16, 16 int8: d = fma(q0*s, x0, 0), d = fma(q_i*s, x_i, d) in element
// order; BF16, 8 elements: d = fma(w0, x0, w1*x1), then
// d = fma(w_2j, x_2j, fma(w_2j+1, x_2j+1, d)) for j = 1..3); the lane adds
// its chunks in order to a sum that starts at 0; the warp reduces with
// __shfl_down (offsets 16..1); split rows add the W warp partials in order
// to 0; the bias is added and the result rounded to BF16.  The helpers below
// compute two independent chunk chains at once (packed FP32x2, FTZ), which
// is the same arithmetic per chain.
__device__ __forceinline__ unsigned long long f2_bits(float2 v) {
  return (static_cast<unsigned long long>(__float_as_uint(v.y)) << 32) |
         __float_as_uint(v.x);
}
__device__ __forceinline__ float2 bits_f2(unsigned long long b) {
  return make_float2(__uint_as_float(uint32_t(b)), __uint_as_float(uint32_t(b >> 32)));
}
__device__ __forceinline__ float2 fma2_ftz(float2 a, float2 b, float2 c) {
  unsigned long long d;
  asm("fma.rn.ftz.f32x2 %0, %1, %2, %3;"
      : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)), "l"(f2_bits(c)));
  return bits_f2(d);
}
__device__ __forceinline__ float2 mul2_ftz(float2 a, float2 b) {
  unsigned long long d;
  asm("mul.rn.ftz.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return bits_f2(d);
}
__device__ __forceinline__ float add_ftz(float a, float b) {
  float d;
  asm("add.rn.ftz.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}
// Exact int8 -> FP32 of byte j of two words (biased by XOR 0x80 first).
template <int kJ>
__device__ __forceinline__ float2 s8_pair(uint32_t b0, uint32_t b1) {
  constexpr uint32_t sel = 0x7540u + kJ;
  return __fadd2_rn(f2(__uint_as_float(__byte_perm(b0, 0x4B000000u, sel)),
                       __uint_as_float(__byte_perm(b1, 0x4B000000u, sel))),
                    f2(-8388736.0f, -8388736.0f));
}
// W8A16: the reference chains of chunk words w0 (chain .x) and w1 (chain .y)
// with x planes x0 / x1 and scales (s0, s1).  One 32-bit word = elements
// 4p..4p+3 of a chunk (plane p).
template <int kP>
__device__ __forceinline__ float2 ref_w8_word(uint32_t w0, uint32_t w1, float4 x0,
                                              float4 x1, float2 sc, float2 d) {
  const uint32_t b0 = w0 ^ 0x80808080u, b1 = w1 ^ 0x80808080u;
  const float2 q0 = mul2_ftz(s8_pair<0>(b0, b1), sc);
  const float2 q1 = mul2_ftz(s8_pair<1>(b0, b1), sc);
  const float2 q2 = mul2_ftz(s8_pair<2>(b0, b1), sc);
  const float2 q3 = mul2_ftz(s8_pair<3>(b0, b1), sc);
  d = fma2_ftz(q0, f2(x0.x, x1.x), d);
  d = fma2_ftz(q1, f2(x0.y, x1.y), d);
  d = fma2_ftz(q2, f2(x0.z, x1.z), d);
  d = fma2_ftz(q3, f2(x0.w, x1.w), d);
  return d;
}
__device__ __forceinline__ float2 ref_w8_chunks(uint4 w0, uint4 w1, const float4* x0,
                                                const float4* x1, float2 sc) {
  float2 d = f2(0.0f, 0.0f);
  d = ref_w8_word<0>(w0.x, w1.x, x0[0], x1[0], sc, d);
  d = ref_w8_word<1>(w0.y, w1.y, x0[1], x1[1], sc, d);
  d = ref_w8_word<2>(w0.z, w1.z, x0[2], x1[2], sc, d);
  d = ref_w8_word<3>(w0.w, w1.w, x0[3], x1[3], sc, d);
  return d;
}
// BF16: the reference chains of two 8-element chunks.
__device__ __forceinline__ float2 ref_bf16_chunks(uint4 w0, uint4 w1, const float4* x0,
                                                  const float4* x1) {
  const float2 wa0 = f2(bf16_lo(w0.x), bf16_lo(w1.x)), wb0 = f2(bf16_hi(w0.x), bf16_hi(w1.x));
  const float2 wa1 = f2(bf16_lo(w0.y), bf16_lo(w1.y)), wb1 = f2(bf16_hi(w0.y), bf16_hi(w1.y));
  const float2 wa2 = f2(bf16_lo(w0.z), bf16_lo(w1.z)), wb2 = f2(bf16_hi(w0.z), bf16_hi(w1.z));
  const float2 wa3 = f2(bf16_lo(w0.w), bf16_lo(w1.w)), wb3 = f2(bf16_hi(w0.w), bf16_hi(w1.w));
  float2 d = mul2_ftz(wb0, f2(x0[0].y, x1[0].y));
  d = fma2_ftz(wa0, f2(x0[0].x, x1[0].x), d);
  d = fma2_ftz(wb1, f2(x0[0].w, x1[0].w), d);
  d = fma2_ftz(wa1, f2(x0[0].z, x1[0].z), d);
  d = fma2_ftz(wb2, f2(x0[1].y, x1[1].y), d);
  d = fma2_ftz(wa2, f2(x0[1].x, x1[1].x), d);
  d = fma2_ftz(wb3, f2(x0[1].w, x1[1].w), d);
  d = fma2_ftz(wa3, f2(x0[1].z, x1[1].z), d);
  return d;
}

constexpr int kConsumerWarps = 16;
constexpr int kBulkSmemBudget = 200 * 1024;
constexpr int kMaxStages = 6;

static __device__ int g_gemv_status = 0;

// Tile geometry.  kWPR == 1: kCW consumer warps x (32 / kLPR) row groups
// per warp x kR rows per lane group; a row is covered by kLPR lanes (16-byte
// chunks c = l, l + kLPR, ...), kLPR chosen per shape so that the chunk
// count divides evenly (896 INT8 = 56 chunks -> 8 lanes); the row groups of
// a warp read the same x words, which shared memory broadcasts.
// kWPR > 1 (small / long-K matrices, to put more SMs on the stream): each
// row is split across kWPR warps of 32 lanes, whose partial sums meet in
// shared memory once per tile.
// kK != 0 compiles the kernel for that in_features (the Qwen2.5 hidden size
// 896): the chunk loop is fully unrolled and every shared-memory offset is
// an immediate.  kK == 0 handles any in_features.
// kRef: the reference summation order above (kLPR == 32, kR == 1).
// kCW: consumer warps (16; 24 for one large-matrix geometry).
template <bool kW8, int kLPR, int kR, int kWPR, int kK, bool kRef, int kCW = kConsumerWarps>
__global__ void __launch_bounds__(32 * (kCW + 1), 1)
gemv_bulk_kernel(const void* __restrict__ weight,
                 const bf16* __restrict__ scales,
                 const bf16* __restrict__ bias,
                 const bf16* __restrict__ input, bf16* __restrict__ output,
                 int n_rows, int k_arg, int stages, int stage_bytes,
                 int w_tile_bytes, float* __restrict__ block_value,
                 int* __restrict__ block_index, const GemvFusion fusion) {
  constexpr int kEPC = kW8 ? 16 : 8;  // elements per 16-byte chunk
  constexpr int kPlanes = kEPC / 4;
  static_assert(kWPR == 1 || (kLPR == 32 && kR == 1), "split rows use whole warps");
  static_assert(!kRef || (kLPR == 32 && kR == 1), "reference order: one row per warp");
  constexpr int kGroups = kWPR > 1 ? 1 : 32 / kLPR;  // row groups per warp
  constexpr int kWarpRows = kGroups * kR;
  constexpr int kTileRows =
      kWPR > 1 ? kCW / kWPR : kCW * kWarpRows;
  extern __shared__ __align__(128) unsigned char smem_bulk[];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int k = kK != 0 ? kK : k_arg;
  const int row_bytes = kW8 ? k : 2 * k;
  const int chunks = k / kEPC;
  const int groups = (k + 63) >> 6;
  const int num_tiles = (n_rows + kTileRows - 1) / kTileRows;
  // Chunk iterations per lane when kK is known (with a bound check if the
  // lanes do not divide the chunks evenly).
  constexpr int kChunks = kK / kEPC;
  constexpr int kSpan = kLPR * kWPR;
  constexpr int kIters = kK != 0 ? (kChunks + kSpan - 1) / kSpan : 0;
  constexpr bool kExact = kK != 0 && kChunks % kSpan == 0;

  float4* xs = reinterpret_cast<float4*>(smem_bulk + size_t(stages) * stage_bytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(xs + (k >> 2));
  const uint32_t bar_full = smem_u32(bars);
  const uint32_t bar_empty = bar_full + 8 * stages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * stages);
  float* red_v = reinterpret_cast<float*>(bars + 2 * stages + 1);
  int* red_i = reinterpret_cast<int*>(red_v + kCW);
  float* red_part = reinterpret_cast<float*>(red_i + kCW);  // [2][warps]
  float* norm_red = red_part + 2 * kCW;                       // [warps]

  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, kCW);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == 0) {
    if (lane == 0) {
      const unsigned char* wbase = static_cast<const unsigned char*>(weight);
      int i = 0, s = 0;
      uint32_t ph = 0;
      for (int tile = blockIdx.x; tile < num_tiles;
           tile += gridDim.x, ++i, s = (s + 1 == stages ? 0 : s + 1),
               ph ^= (s == 0 ? 1u : 0u)) {
        if (!mbar_wait_bounded(bar_empty + 8 * s, ph ^ 1, abort_flag,
                               B200_DEVICE_TIMEOUT_PIPELINE, &g_gemv_status))
          break;
        const int row0 = tile * kTileRows;
        const int rows = min(kTileRows, n_rows - row0);
        const uint32_t wbytes = uint32_t(rows) * row_bytes;
        const uint32_t sbytes = kW8 ? uint32_t(rows) * groups * 2 : 0u;
        unsigned char* st = smem_bulk + size_t(s) * stage_bytes;
        mbar_arrive_expect_tx(bar_full + 8 * s, wbytes + sbytes);
        bulk_load(smem_u32(st), wbase + size_t(row0) * row_bytes, wbytes,
                  bar_full + 8 * s);
        if (kW8) {
          bulk_load(smem_u32(st + w_tile_bytes), scales + size_t(row0) * groups,
                    sbytes, bar_full + 8 * s);
        }
      }
    }
  } else {
    // ------------------------------------------------------------ consumers
    const int ct = threadIdx.x - 32;
    pdl_wait_primary();
    float norm_scale = 1.0f;
    if (fusion.in_mode == 1) {
      // RMSNorm of the input: FP32 sum of squares over the consumer threads.
      float ss = 0.0f;
      for (int e4 = ct; e4 < (k >> 2); e4 += kCW * 32) {
        const uint2 raw = reinterpret_cast<const uint2*>(input)[e4];
        const float a = bf16_lo(raw.x), b = bf16_hi(raw.x);
        const float c = bf16_lo(raw.y), d = bf16_hi(raw.y);
        ss = fmaf(a, a, ss);
        ss = fmaf(b, b, ss);
        ss = fmaf(c, c, ss);
        ss = fmaf(d, d, ss);
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
      if (lane == 0) norm_red[warp - 1] = ss;
      asm volatile("bar.sync 1, %0;" ::"r"(kCW * 32) : "memory");
      float total = 0.0f;
#pragma unroll
      for (int w = 0; w < kCW; ++w) total += norm_red[w];
      norm_scale = rsqrtf(total / float(k) + fusion.eps);
    }
    // x -> FP32 planes: xs[p * chunks + c] = x[c*kEPC + 4p .. +3].
    for (int e4 = ct; e4 < (k >> 2); e4 += kCW * 32) {
      const uint2 raw = reinterpret_cast<const uint2*>(input)[e4];
      const int c = (e4 * 4) / kEPC;
      const int p = ((e4 * 4) % kEPC) >> 2;
      float4 v = make_float4(bf16_lo(raw.x), bf16_hi(raw.x), bf16_lo(raw.y),
                             bf16_hi(raw.y));
      if (fusion.in_mode == 1) {
        const uint2 wr = reinterpret_cast<const uint2*>(fusion.norm_w)[e4];
        v.x = bf16_round(v.x * bf16_lo(wr.x) * norm_scale);
        v.y = bf16_round(v.y * bf16_hi(wr.x) * norm_scale);
        v.z = bf16_round(v.z * bf16_lo(wr.y) * norm_scale);
        v.w = bf16_round(v.w * bf16_hi(wr.y) * norm_scale);
      } else if (fusion.in_mode == 2) {
        const uint2 ur = reinterpret_cast<const uint2*>(input + k)[e4];
        v.x = bf16_round(v.x / (1.0f + expf(-v.x)) * bf16_lo(ur.x));
        v.y = bf16_round(v.y / (1.0f + expf(-v.y)) * bf16_hi(ur.x));
        v.z = bf16_round(v.z / (1.0f + expf(-v.z)) * bf16_lo(ur.y));
        v.w = bf16_round(v.w / (1.0f + expf(-v.w)) * bf16_hi(ur.y));
      }
      xs[p * chunks + c] = v;
    }
    asm volatile("bar.sync 1, %0;" ::"r"(kCW * 32) : "memory");

    const int cw = warp - 1;                  // consumer warp index
    const int gl = lane / kLPR;               // row group within the warp
    const int ll = lane % kLPR;               // lane within the row group
    const int ksub = kWPR > 1 ? cw % kWPR : 0;  // K slice of a split row
    const int rloc0 =
        kWPR > 1 ? cw / kWPR : cw * kWarpRows + gl * kR;
    float best = -FLT_MAX;
    int best_index = INT_MAX;
    int i = 0, s = 0;
    uint32_t ph = 0;
    for (int tile = blockIdx.x; tile < num_tiles;
         tile += gridDim.x, ++i, s = (s + 1 == stages ? 0 : s + 1),
             ph ^= (s == 0 ? 1u : 0u)) {
      // Warp-uniform outcome.  Split rows (kWPR > 1) meet at a named barrier
      // every tile, so a failed wait must not make a warp leave the loop
      // early: it skips the work instead (later waits fail at once once the
      // abort flag is up).
      const bool ok = __all_sync(
          0xffffffffu, mbar_wait_bounded(bar_full + 8 * s, ph, abort_flag,
                                         B200_DEVICE_TIMEOUT_PIPELINE, &g_gemv_status));
      if (!ok && kWPR == 1) break;
      const unsigned char* wt = smem_bulk + size_t(s) * stage_bytes;
      const bf16* stile = reinterpret_cast<const bf16*>(wt + w_tile_bytes);
      float2 acc2[kR];
#pragma unroll
      for (int r = 0; r < kR; ++r) acc2[r] = f2(0.0f, 0.0f);
      auto chunk_step = [&](int c) {
        float4 xv[kPlanes];
#pragma unroll
        for (int p = 0; p < kPlanes; ++p) xv[p] = xs[p * chunks + c];
#pragma unroll
        for (int r = 0; r < kR; ++r) {
          const uint4 wv = *reinterpret_cast<const uint4*>(
              wt + (rloc0 + r) * row_bytes + c * 16);
          if constexpr (kW8) {
            // Two independent chains of the chunk's 16 products, each then
            // scaled into the row accumulator with one packed FMA.
            float2 a = f2(0.0f, 0.0f);
            float2 b = f2(0.0f, 0.0f);
            a = dot4_s8_x2(wv.x, xv[0], a);
            b = dot4_s8_x2(wv.y, xv[1], b);
            a = dot4_s8_x2(wv.z, xv[2], a);
            b = dot4_s8_x2(wv.w, xv[3], b);
            const float sc =
                __bfloat162float(stile[(rloc0 + r) * groups + (c >> 2)]);
            acc2[r] = __ffma2_rn(a, f2(sc, sc), acc2[r]);
            acc2[r] = __ffma2_rn(b, f2(sc, sc), acc2[r]);
          } else {
            acc2[r] = dot4_bf16_x2(wv.x, wv.y, xv[0], acc2[r]);
            acc2[r] = dot4_bf16_x2(wv.z, wv.w, xv[1], acc2[r]);
          }
        }
      };
      const int c0 = ok ? ksub * kLPR + ll : chunks;  // failed: no chunks
      float ref_sum = 0.0f;
      if constexpr (kRef) {
        // Chunks c0, c0 + kSpan, ... in pairs; the lane sum adds them in order.
        const int rl = rloc0;
        for (int c = c0; c < chunks; c += 2 * kSpan) {
          const int c1 = c + kSpan < chunks ? c + kSpan : c;
          float4 x0[kPlanes], x1[kPlanes];
#pragma unroll
          for (int p = 0; p < kPlanes; ++p) {
            x0[p] = xs[p * chunks + c];
            x1[p] = xs[p * chunks + c1];
          }
          const uint4 w0 = *reinterpret_cast<const uint4*>(wt + rl * row_bytes + c * 16);
          const uint4 w1 = *reinterpret_cast<const uint4*>(wt + rl * row_bytes + c1 * 16);
          float2 d;
          if constexpr (kW8) {
            const float2 sc = f2(__bfloat162float(stile[rl * groups + (c >> 2)]),
                                 __bfloat162float(stile[rl * groups + (c1 >> 2)]));
            d = ref_w8_chunks(w0, w1, x0, x1, sc);
          } else {
            d = ref_bf16_chunks(w0, w1, x0, x1);
          }
          ref_sum = add_ftz(ref_sum, d.x);
          if (c1 != c) ref_sum = add_ftz(ref_sum, d.y);
        }
      } else if constexpr (kK != 0) {
#pragma unroll
        for (int j = 0; j < kIters; ++j) {
          const int c = c0 + j * kSpan;
          if ((kExact && ok) || c < kChunks) chunk_step(c);
        }
      } else {
#pragma unroll 2
        for (int c = c0; c < chunks; c += kSpan) chunk_step(c);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_empty + 8 * s);
      const int row0 = tile * kTileRows + rloc0;
#pragma unroll
      for (int r = 0; r < kR; ++r) {
        float v;
        if constexpr (kRef) {
          // Same tree as the reference's __shfl_down reduction at lane 0.
          v = ref_sum;
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) {
            v = add_ftz(v, __shfl_xor_sync(0xffffffffu, v, off));
          }
        } else {
          v = acc2[r].x + acc2[r].y;
#pragma unroll
          for (int off = kLPR / 2; off > 0; off >>= 1) {
            v += __shfl_xor_sync(0xffffffffu, v, off);
          }
        }
        if constexpr (kWPR > 1) {
          // Partials of the kWPR warps of a row meet in shared memory
          // (double-buffered by tile parity: one barrier per tile).
          float* part = red_part + (i & 1) * kCW;
          if (lane == 0) part[cw] = v;
          asm volatile("bar.sync 1, %0;" ::"r"(kCW * 32) : "memory");
          if (ksub == 0) {
            v = 0.0f;
#pragma unroll
            for (int j = 0; j < kWPR; ++j) {
              v = kRef ? add_ftz(v, part[cw + j]) : v + part[cw + j];
            }
          }
        }
        const int row = row0 + r;
        if (ok && ll == 0 && ksub == 0 && row < n_rows) {
          const float b = bias ? __bfloat162float(bias[row]) : 0.0f;
          const bf16 y = __float2bfloat16_rn(kRef ? add_ftz(v, b) : v + b);
          if (fusion.residual != nullptr) {
            fusion.residual[row] = __float2bfloat16_rn(
                __bfloat162float(fusion.residual[row]) + __bfloat162float(y));
          } else {
            output[row] = y;
          }
          argmax_update(best, best_index, __bfloat162float(y), row);
        }
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
        red_v[warp - 1] = best;
        red_i[warp - 1] = best_index;
      }
      asm volatile("bar.sync 1, %0;" ::"r"(kCW * 32) : "memory");
      if (ct == 0) {
        float b = -FLT_MAX;
        int bi = INT_MAX;
        for (int w = 0; w < kCW; ++w) argmax_update(b, bi, red_v[w], red_i[w]);
        block_value[blockIdx.x] = b;
        block_index[blockIdx.x] = bi;
      }
    }
  }
  __syncthreads();
}

struct BulkPlan {
  int lpr = 0;  // lanes per row (0: plan not possible)
  int r = 0;    // rows per lane group
  int wpr = 1;  // warps per row
  int stages = 0;
  int stage_bytes = 0;
  int w_tile_bytes = 0;
  int smem = 0;
  int grid = 0;
  bool ref = false;  // reference summation order (kLPR 32, kR 1)
  int cw = kConsumerWarps;  // consumer warps per CTA
};

// SM count of the current device, looked up once per device (a host-side
// cost paid on every GEMV call otherwise).
int device_sm_count() {
  static std::atomic<int> cached[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64) {
    const int c = cached[dev].load(std::memory_order_relaxed);
    if (c > 0) return c;
  }
  int count = 148;
  cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev);
  if (dev >= 0 && dev < 64) cached[dev].store(count, std::memory_order_relaxed);
  return count;
}

// Raises a kernel's dynamic shared-memory limit to the bulk budget once per
// device (every plan stays below it).
template <auto kKernel>
cudaError_t bulk_smem_attr() {
  static std::atomic<unsigned long long> done{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = dev >= 0 && dev < 64 ? 1ull << dev : 0ull;
  if (bit != 0 && (done.load(std::memory_order_acquire) & bit) != 0) return cudaSuccess;
  const cudaError_t e = cudaFuncSetAttribute(
      kKernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kBulkSmemBudget + 8 * 1024);
  if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_release);
  return e;
}

// Chooses the tile geometry (tiles of at least min_rows rows) by a simple
// cost model: bytes streamed by the busiest SM (waves x tile bytes), divided
// by the fraction of lanes doing useful work in the chunk loop (idle lanes
// still cost issue slots, which bound the INT8 path), plus a small charge
// per tile for the cross-warp reduction of split rows.  Large matrices get
// rows whose chunks divide evenly among the lanes (896 INT8 -> 8 lanes);
// small or long-K ones get split rows that reach every SM.
BulkPlan plan_bulk(bool w8, int n, int k, int min_rows, int table_lpr = 0, int table_r = 0,
                   int table_wpr = 0) {
  BulkPlan best;
  double best_cost = 1e30;
  const int sms = device_sm_count();
  const int row_bytes = w8 ? k : 2 * k;
  const int groups = (k + 63) / 64;
  const int chunks = w8 ? k / 16 : k / 8;
  const int x_bytes = k * 4;
  const int budget = kBulkSmemBudget - x_bytes - 512;
  struct Cand { int lpr, r, wpr, cw; };
  // The last candidate (24 consumer warps, 96-row tiles) serves only large
  // W8 matrices at in_features 896: 896 -> 151936 in 26.0 vs 27.2 us (more
  // warps hide the shared-memory load latency); the smaller shapes measured
  // slower with 24 warps.
  const Cand cands[] = {{8, 2, 1, 16}, {8, 1, 1, 16}, {16, 2, 1, 16}, {16, 1, 1, 16},
                        {32, 4, 1, 16}, {32, 2, 1, 16}, {32, 1, 1, 16}, {32, 1, 2, 16},
                        {32, 1, 4, 16}, {16, 2, 1, 24}};
  // B200_GEMV_PLAN=lpr,r,wpr restricts the choice to that geometry (tuning).
  int force_lpr = table_lpr, force_r = table_r, force_wpr = table_wpr;
  if (const char* e = getenv("B200_GEMV_PLAN")) {
    sscanf(e, "%d,%d,%d", &force_lpr, &force_r, &force_wpr);
  }
  for (const Cand& c : cands) {
    if (force_lpr > 0 && (c.lpr != force_lpr || c.r != force_r || c.wpr != force_wpr)) continue;
    if (c.cw != kConsumerWarps && !(w8 && k == 896 && n >= 16384)) continue;
    const int rows = c.wpr > 1 ? c.cw / c.wpr : c.cw * (32 / c.lpr) * c.r;
    if (rows < min_rows) continue;
    // Each tile's scale rows are one 1-D bulk copy: its source offset
    // (row0 * groups * 2 bytes) must stay 16-byte aligned.
    if (w8 && (rows * groups * 2) % 16 != 0) continue;
    const int wt = rows * row_bytes;
    const int st = (wt + (w8 ? rows * groups * 2 : 0) + 127) / 128 * 128;
    const int stages = budget / st < kMaxStages ? budget / st : kMaxStages;
    if (stages < 2) continue;
    const int span = c.lpr * c.wpr;
    const int iters = (chunks + span - 1) / span;
    const double eff = double(chunks) / double(iters * span);
    const int tiles = (n + rows - 1) / rows;
    const int waves = (tiles + sms - 1) / sms;
    // Large W8 matrices at in_features 896: two rows per lane (16 lanes a
    // row) measured 2.7% faster than one (27.6 vs 28.4 us on 896 -> 151936)
    // although a lane's 3.5 chunks leave lanes idle; 32 lanes with x in
    // registers, or 4 rows a lane, measured slower (32-40 us).
    const double shape_factor =
        (w8 && k == 896 && n >= 16384 && !(c.lpr == 16 && c.r == 2)) ? 1.2 : 1.0;
    const double cost = double(waves) * rows * row_bytes / eff * shape_factor +
                        (c.wpr > 1 ? waves * 2048.0 : 0.0);
    if (cost < best_cost * 0.999) {
      best_cost = cost;
      best.lpr = c.lpr;
      best.r = c.r;
      best.wpr = c.wpr;
      best.stages = stages;
      best.stage_bytes = st;
      best.w_tile_bytes = wt;
      best.smem = stages * st + x_bytes + 8 * 2 * stages + 8 + 8 * c.cw + 8 * c.cw + 4 * c.cw;
      best.cw = c.cw;
      best.grid = tiles < sms ? tiles : sms;
    }
  }
  return best;
}

// Reference-order plan: one warp per row (the row split over 4 warps when
// the reference splits it: a GEMV with in_features > 1024), 16 or 4 rows per
// tile, as many stages as fit.
BulkPlan plan_bulk_ref(bool w8, int n, int k, bool lm_head) {
  BulkPlan p;
  const int sms = device_sm_count();
  const int wpr = (k > 1024 && (w8 || !lm_head)) ? 4 : 1;
  const int rows = kConsumerWarps / wpr;
  const int row_bytes = w8 ? k : 2 * k;
  const int groups = (k + 63) / 64;
  const int budget = kBulkSmemBudget - k * 4 - 512;
  const int st = (rows * row_bytes + (w8 ? rows * groups * 2 : 0) + 127) / 128 * 128;
  const int stages = budget / st < 16 ? budget / st : 16;
  if (stages < 2) return p;
  // 16-byte aligned scale copies per tile (4-row tiles need an even group
  // count); otherwise no reference-order plan (the call takes the fast one).
  if (w8 && (rows * groups * 2) % 16 != 0) return p;
  const int tiles = (n + rows - 1) / rows;
  int grid = tiles < sms ? tiles : sms;
  if (lm_head && grid > (n + 7) / 8) grid = (n + 7) / 8;  // ceil(n/8) partials
  p.lpr = 32;
  p.r = 1;
  p.wpr = wpr;
  p.stages = stages;
  p.stage_bytes = st;
  p.w_tile_bytes = rows * row_bytes;
  p.smem = stages * st + k * 4 + 8 * 2 * stages + 8 + 8 * kConsumerWarps +
           8 * kConsumerWarps + 4 * kConsumerWarps;
  p.grid = grid;
  p.ref = true;
  return p;
}

template <bool kW8, int kLPR, int kR, int kWPR, bool kRef = false, int kCW = kConsumerWarps>
cudaError_t launch_bulk(const BulkPlan& p, const void* w, const bf16* s,
                        const bf16* b, const bf16* x, bf16* y, int n, int k,
                        float* bv, int* bi, cudaStream_t stream,
                        const GemvFusion& fusion) {
  auto kernel = k == 896 ? gemv_bulk_kernel<kW8, kLPR, kR, kWPR, 896, kRef, kCW>
                         : gemv_bulk_kernel<kW8, kLPR, kR, kWPR, 0, kRef, kCW>;
  cudaError_t e = k == 896
                      ? bulk_smem_attr<gemv_bulk_kernel<kW8, kLPR, kR, kWPR, 896, kRef, kCW>>()
                      : bulk_smem_attr<gemv_bulk_kernel<kW8, kLPR, kR, kWPR, 0, kRef, kCW>>();
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(32 * (kCW + 1));
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, w, s, b, x, y, n, k, p.stages,
                            p.stage_bytes, p.w_tile_bytes, bv, bi, fusion);
}

template <bool kW8>
cudaError_t dispatch_bulk(const BulkPlan& p, const void* w, const bf16* s,
                          const bf16* b, const bf16* x, bf16* y, int n, int k,
                          float* bv, int* bi, cudaStream_t st, const GemvFusion& f) {
  if (p.ref) {
    return p.wpr == 4
               ? launch_bulk<kW8, 32, 1, 4, true>(p, w, s, b, x, y, n, k, bv, bi, st, f)
               : launch_bulk<kW8, 32, 1, 1, true>(p, w, s, b, x, y, n, k, bv, bi, st, f);
  }
  if constexpr (kW8) {
    if (p.cw == 24) return launch_bulk<true, 16, 2, 1, false, 24>(p, w, s, b, x, y, n, k, bv, bi, st, f);
  }
  if (p.wpr == 4) return launch_bulk<kW8, 32, 1, 4>(p, w, s, b, x, y, n, k, bv, bi, st, f);
  if (p.wpr == 2) return launch_bulk<kW8, 32, 1, 2>(p, w, s, b, x, y, n, k, bv, bi, st, f);
  if (p.lpr == 8) {
    return p.r == 2 ? launch_bulk<kW8, 8, 2, 1>(p, w, s, b, x, y, n, k, bv, bi, st, f)
                    : launch_bulk<kW8, 8, 1, 1>(p, w, s, b, x, y, n, k, bv, bi, st, f);
  }
  if (p.lpr == 16) {
    return p.r == 2 ? launch_bulk<kW8, 16, 2, 1>(p, w, s, b, x, y, n, k, bv, bi, st, f)
                    : launch_bulk<kW8, 16, 1, 1>(p, w, s, b, x, y, n, k, bv, bi, st, f);
  }
  if (p.r == 4) return launch_bulk<kW8, 32, 4, 1>(p, w, s, b, x, y, n, k, bv, bi, st, f);
  return p.r == 2 ? launch_bulk<kW8, 32, 2, 1>(p, w, s, b, x, y, n, k, bv, bi, st, f)
                  : launch_bulk<kW8, 32, 1, 1>(p, w, s, b, x, y, n, k, bv, bi, st, f);
}

struct GemvConfig {
  int tpr;  // threads per team
  int r;    // rows per team
};

// Shape heuristic: large matrices (more 16-byte chunks than ~8 per thread of
// a full B200) use 4 rows per team to amortise x; everything else spreads the
// matrix over as many threads as possible, <= 2 chunk columns per thread.
GemvConfig choose_config(int n_rows, int chunks, bool lm_head) {
  const long long total = (long long)n_rows * chunks;
  const bool big = total >= 148LL * 2048 * 4;
  const int r = big ? 4 : 1;
  const int per_thread = big ? 8 : 2;
  int want = (chunks + per_thread - 1) / per_thread;
  int tpr = 4;
  while (tpr < want && tpr < 256) tpr <<= 1;
  if (lm_head && tpr > 32) tpr = 32;
  return {tpr, r};
}

template <bool kW8, int kTPR, int kR>
cudaError_t launch_stream(const void* w, const bf16* s, const bf16* b,
                          const bf16* x, bf16* y, int n, int k, float* bv,
                          int* bi, cudaStream_t stream, int* grid_out) {
  constexpr int kRowsPerBlock = (kThreads / kTPR) * kR;
  const int grid = (n + kRowsPerBlock - 1) / kRowsPerBlock;
  const size_t smem = size_t(k) * 2;
  auto kernel = gemv_stream_kernel<kW8, kTPR, kR>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(
        kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
  }
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
  if (grid_out) *grid_out = grid;
  return cudaLaunchKernelEx(&cfg, kernel, w, s, b, x, y, n, k, bv, bi);
}

template <bool kW8, int kR>
cudaError_t dispatch_tpr(int tpr, const void* w, const bf16* s, const bf16* b,
                         const bf16* x, bf16* y, int n, int k, float* bv,
                         int* bi, cudaStream_t st, int* grid) {
  switch (tpr) {
    case 4: return launch_stream<kW8, 4, kR>(w, s, b, x, y, n, k, bv, bi, st, grid);
    case 8: return launch_stream<kW8, 8, kR>(w, s, b, x, y, n, k, bv, bi, st, grid);
    case 16: return launch_stream<kW8, 16, kR>(w, s, b, x, y, n, k, bv, bi, st, grid);
    case 32: return launch_stream<kW8, 32, kR>(w, s, b, x, y, n, k, bv, bi, st, grid);
    case 64: return launch_stream<kW8, 64, kR>(w, s, b, x, y, n, k, bv, bi, st, grid);
    case 128: return launch_stream<kW8, 128, kR>(w, s, b, x, y, n, k, bv, bi, st, grid);
    default: return launch_stream<kW8, 256, kR>(w, s, b, x, y, n, k, bv, bi, st, grid);
  }
}

template <bool kW8>
cudaError_t launch_generic(const void* w, const bf16* s, const bf16* b,
                           const bf16* x, bf16* y, int n, int k, float* bv,
                           int* bi, cudaStream_t stream, int* grid_out) {
  const int grid = (n + 7) / 8;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (grid_out) *grid_out = grid;
  return cudaLaunchKernelEx(&cfg, gemv_generic_kernel<kW8>, w, s, b, x, y, n,
                            k, bv, bi);
}

bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

}  // namespace

bool gemv_uses_fast_path(bool w8, const void* weight, const void* input,
                         int k) {
  const int elems_per_chunk = w8 ? 16 : 8;
  return k > 0 && k % elems_per_chunk == 0 && k <= 98304 &&
         aligned16(weight) && aligned16(input);
}

namespace {

// Which kernel a call runs and with what geometry; computed before any
// launch so that callers with a fixed-size partials buffer can check the
// grid first (b200_lm_head_bf16_noalloc).
struct GemvPlan {
  int kind = 0;  // 0: nothing to do, 1: generic, 2: TMA bulk, 3: stream, 4: i8 MMA
  BulkPlan bulk;
  GemvConfig cfg{0, 0};
  int grid = 0;
};

int stream_rows_per_block(int tpr, int r) { return (kThreads / tpr) * r; }

// The reference's own fast-path conditions (src/cuda/kernels.cu:1540-1579,
// 1627-1655): outside them it runs other kernels, whose order the reference
// mode does not reproduce.
bool reference_fast_shape(bool w8, const void* weight, const void* input, int k,
                          bool lm_head) {
  if (!aligned16(weight) || !aligned16(input)) return false;
  if (w8) return k >= 16 && k % 64 == 0;
  return lm_head ? k % 8 == 0 && k > 0 : k >= 8 && k % 8 == 0;
}

// The integer-tensor-core W8A16 GEMV (gemv_i8tc.cu): B200_GEMV_I8TC=1
// selects it (read at every call).
bool use_i8tc() {
  const char* e = getenv("B200_GEMV_I8TC");
  return e != nullptr && strcmp(e, "1") == 0;
}

GemvPlan plan_gemv(bool w8, const void* weight, const bf16* scales, int n,
                   int k, const void* input, bool lm_head, bool fused = false) {
  GemvPlan plan;
  if (n <= 0) return plan;
  if (w8 && !fused && summation_order() == B200_ORDER_FAST && use_i8tc() &&
      gemv_i8tc_supported(weight, input, scales, n, k)) {
    plan.kind = 4;
    plan.grid = gemv_i8tc_grid(n);
    return plan;
  }
  if (!fused && summation_order() == B200_ORDER_REFERENCE &&
      reference_fast_shape(w8, weight, input, k, lm_head) && n % 8 == 0 &&
      (!w8 || aligned16(scales)) && k <= 32768) {
    plan.bulk = plan_bulk_ref(w8, n, k, lm_head);
    if (plan.bulk.lpr > 0) {
      plan.kind = 2;
      plan.grid = plan.bulk.grid;
      return plan;
    }
  }
  if (!gemv_uses_fast_path(w8, weight, input, k)) {
    plan.kind = 1;
    plan.grid = (n + 7) / 8;
    return plan;
  }
  // Small matrices (<= 2 MB, plain calls): the register-streaming kernel,
  // measured faster than the TMA-ring kernel there (BF16 896 -> 896: 1.45 vs
  // 1.83 us; 896 -> 128: 1.29 vs 1.60 us; W8A16 896 -> 896: 1.81 vs 1.98 us).
  const double mat_bytes = double(n) * k * (w8 ? 1 : 2);
  const bool plain = !fused && !lm_head && getenv("B200_GEMV_PLAN") == nullptr;
  if (plain && mat_bytes <= 2.0 * 1024 * 1024) {
    const int chunks = w8 ? k / 16 : k / 8;
    plan.kind = 3;
    plan.cfg = choose_config(n, chunks, lm_head);
    const int rows = stream_rows_per_block(plan.cfg.tpr, plan.cfg.r);
    plan.grid = (n + rows - 1) / rows;
    return plan;
  }
  // Measured geometry for the Qwen2.5 MLP shape 896 -> 4864 (the cost model
  // below picks 16-row tiles there): W8A16 8 lanes x 1 row, 2.70 vs 3.00 us;
  // BF16 16 lanes x 1 row, 3.05 vs 4.05 us.
  int t_lpr = 0, t_r = 0, t_wpr = 0;
  if (plain && k == 896 && n == 4864) {
    t_lpr = w8 ? 8 : 16;
    t_r = 1;
    t_wpr = 1;
  }
  // TMA-bulk path: needs whole 8-row tiles of 16-byte multiples (n % 8) and
  // 16-byte aligned scales.
  if (n % 8 == 0 && (!w8 || aligned16(scales))) {
    // The LM-head form writes one argmax partial per CTA into a workspace of
    // ceil(n / 8) entries: tiles of >= 8 rows keep the grid within it.
    plan.bulk = plan_bulk(w8, n, k, lm_head ? 8 : 1, t_lpr, t_r, t_wpr);
    if (plan.bulk.lpr > 0) {
      plan.kind = 2;
      plan.grid = plan.bulk.grid;
      return plan;
    }
  }
  const int chunks = w8 ? k / 16 : k / 8;
  plan.kind = 3;
  plan.cfg = choose_config(n, chunks, lm_head);
  const int rows = stream_rows_per_block(plan.cfg.tpr, plan.cfg.r);
  plan.grid = (n + rows - 1) / rows;
  return plan;
}

}  // namespace

namespace {
// -1: not read yet from B200_SUMMATION_ORDER.
std::atomic<int> g_summation_order{-1};
}  // namespace

int summation_order() {
  int v = g_summation_order.load(std::memory_order_relaxed);
  if (v < 0) {
    const char* e = getenv("B200_SUMMATION_ORDER");
    v = (e != nullptr && strcmp(e, "reference") == 0) ? B200_ORDER_REFERENCE
                                                      : B200_ORDER_FAST;
    int expected = -1;
    g_summation_order.compare_exchange_strong(expected, v);
    v = g_summation_order.load(std::memory_order_relaxed);
  }
  return v;
}

void set_summation_order(int order) {
  g_summation_order.store(order, std::memory_order_relaxed);
}

int gemv_grid(bool w8, const void* weight, const bf16* scales,
              const void* input, int n, int k, bool lm_head) {
  return plan_gemv(w8, weight, scales, n, k, input, lm_head).grid;
}

cudaError_t launch_gemv(bool w8, const void* weight, const bf16* scales,
                        const bf16* bias, const bf16* input, bf16* output,
                        int n, int k, float* block_value, int* block_index,
                        cudaStream_t stream, int* grid_out,
                        const GemvFusion* fusion) {
  const GemvFusion nofusion;
  const GemvFusion& f = fusion ? *fusion : nofusion;
  const bool fused = fusion != nullptr &&
                     (f.in_mode != 0 || f.residual != nullptr);
  const GemvPlan plan =
      plan_gemv(w8, weight, scales, n, k, input, block_value != nullptr, fused);
  if (grid_out) *grid_out = plan.grid;
  if (plan.kind == 0) return cudaSuccess;
  // The fusions exist only in the TMA-bulk kernel.
  if (fused && plan.kind != 2) return cudaErrorNotSupported;
  if (plan.kind == 1) {
    return w8 ? launch_generic<true>(weight, scales, bias, input, output, n, k,
                                     block_value, block_index, stream, nullptr)
              : launch_generic<false>(weight, scales, bias, input, output, n,
                                      k, block_value, block_index, stream,
                                      nullptr);
  }
  if (plan.kind == 4) {
    return launch_gemv_i8tc(weight, scales, bias, input, output, n, k, block_value,
                            block_index, stream, nullptr);
  }
  if (plan.kind == 2) {
    const BulkPlan& p = plan.bulk;
    return w8 ? dispatch_bulk<true>(p, weight, scales, bias, input, output, n,
                                    k, block_value, block_index, stream, f)
              : dispatch_bulk<false>(p, weight, scales, bias, input, output,
                                     n, k, block_value, block_index, stream, f);
  }
  const GemvConfig c = plan.cfg;
  if (w8) {
    return c.r == 4 ? dispatch_tpr<true, 4>(c.tpr, weight, scales, bias, input,
                                            output, n, k, block_value,
                                            block_index, stream, nullptr)
                    : dispatch_tpr<true, 1>(c.tpr, weight, scales, bias, input,
                                            output, n, k, block_value,
                                            block_index, stream, nullptr);
  }
  return c.r == 4 ? dispatch_tpr<false, 4>(c.tpr, weight, scales, bias, input,
                                           output, n, k, block_value,
                                           block_index, stream, nullptr)
                  : dispatch_tpr<false, 1>(c.tpr, weight, scales, bias, input,
                                           output, n, k, block_value,
                                           block_index, stream, nullptr);
}

cudaError_t read_gemv_status(int* value, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(value, g_gemv_status, sizeof(int));
  if (e != cudaSuccess || !clear) return e;
  const int zero = 0;
  return cudaMemcpyToSymbol(g_gemv_status, &zero, sizeof(int));
}

cudaError_t launch_argmax_partials(const float* block_value,
                                   const int* block_index, int count,
                                   int* argmax, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(1024);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, argmax_partials_kernel, block_value,
                            block_index, count, argmax);
}

cudaError_t launch_argmax_bf16(const bf16* values, int n, int* out,
                               cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(1024);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, argmax_bf16_kernel, values, n, out);
}

}  // namespace b200
