// Causal GQA prefill attention on the tensor cores (head_dim 64).
//
// Replaces, for the native engine's prefill, the one-CTA-per-(head, token)
// CUDA-core kernel (the reference's attention_prefill_bf16_kernel,
// src/cuda/kernels.cu:221-283, has the same structure).  One CTA per (head,
// 128-query tile) walks the key blocks of 128 positions up to its last query:
//   S = Q K^T    tcgen05.mma (M=128 queries, N=128 keys, K=64), FP32 in TMEM;
//   softmax      one thread per query row (warps 0..3 = TMEM lane quarters):
//                tcgen05.ld of its S row, scale, causal mask, online
//                maximum / sum, P = exp(S - max) rounded to BF16 and written
//                back into TMEM with tcgen05.st;
//   O_j = P V    tcgen05.mma with A = P FROM TENSOR MEMORY (M=128, K=128
//                keys) and B = V^T from shared memory (N=64, K-major), FP32
//                in TMEM; the row thread reads O_j and folds it into its
//                register accumulator with the online-softmax rescale.
// Output: bf16(O / l) per query row.  Arithmetic: FP32 scores and sums as
// the reference, with P rounded to BF16 for the P.V product (the tensor
// cores take BF16 operands), so results agree within the attention
// tolerance rather than bit for bit.
//
// Operands are staged by the CTA's threads with plain 16-byte loads into the
// 128-byte-swizzled K-major layouts (Q, K: row = query / key, 64 dims =
// 128 B; V^T: row = dim, two 64-key sub-tiles).  Key blocks are processed
// one after another (the MMAs, the softmax and the next block's staging do
// not overlap); waits are bounded and report B200_DEVICE_TIMEOUT_PIPELINE.
#include <cfloat>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace b200 {

__device__ int g_att_status = 0;

cudaError_t read_att_status(int* value, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(value, g_att_status, sizeof(int));
  if (e != cudaSuccess || !clear) return e;
  const int zero = 0;
  return cudaMemcpyToSymbol(g_att_status, &zero, sizeof(int));
}

namespace {

constexpr int kQ = 128;         // queries per CTA
constexpr int kKeys = 128;      // keys per block
constexpr int kD = 64;          // head dim
constexpr int kThreads = 256;
constexpr int kQBytes = kQ * kD * 2;      // 16 KB
constexpr int kKBytes = kKeys * kD * 2;   // 16 KB
constexpr int kVBytes = kD * kKeys * 2;   // 16 KB (two [64 x 64] sub-tiles)
constexpr int kSmem = 1024 + kQBytes + kKBytes + kVBytes + 64;
// TMEM columns: S [0,128), P [128,192) (BF16 pairs), O [192,256)
constexpr uint32_t kColS = 0, kColP = 128, kColO = 192;

__device__ __forceinline__ int sw(int r, int c) {  // byte offset, [rows x 64] BF16, SW128
  return r * 128 + ((((c >> 3) ^ (r & 7))) << 4) + (c & 7) * 2;
}

__device__ __forceinline__ bool wait_a(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  return mbar_wait_bounded(bar, parity, abort_flag, B200_DEVICE_TIMEOUT_PIPELINE, &g_att_status);
}

__global__ void __launch_bounds__(kThreads, 1)
attention_prefill_tc_kernel(const bf16* __restrict__ q, int q_stride, const bf16* __restrict__ kcache,
                            const bf16* __restrict__ vcache, bf16* __restrict__ out, int out_stride,
                            int tokens, int pos0, int heads, int kv_heads, int max_seq) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* qs = smem;
  unsigned char* ks = qs + kQBytes;
  unsigned char* vs = ks + kKBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(vs + kVBytes);
  const uint32_t bar_s = smem_u32(bars), bar_p = bar_s + 8, bar_o = bar_s + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int head = blockIdx.x;
  const int q0 = blockIdx.y * kQ;
  const int kvh = head / (heads / kv_heads);
  const int warp = threadIdx.x >> 5;
  const bf16* kb = kcache + size_t(kvh) * max_seq * kD;
  const bf16* vb = vcache + size_t(kvh) * max_seq * kD;

  if (threadIdx.x == 0) {
    mbar_init(bar_s, 1);
    mbar_init(bar_p, 128);
    mbar_init(bar_o, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 4) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(256)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  pdl_launch_dependents();
  pdl_wait_primary();
  // Q tile: 128 rows x 8 chunks of 16 B; rows past the prompt are zero.
  for (int i = threadIdx.x; i < kQ * 8; i += kThreads) {
    const int r = i >> 3, c = (i & 7) * 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (q0 + r < tokens) {
      v = *reinterpret_cast<const uint4*>(q + size_t(q0 + r) * q_stride + head * kD + c);
    }
    *reinterpret_cast<uint4*>(qs + sw(r, c)) = v;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Row state (warps 0..3: thread = query row q0 + threadIdx.x).
  const int row = threadIdx.x;
  const int qpos = pos0 + q0 + row;  // this query's position
  float m_run = -FLT_MAX, l_run = 0.0f;
  float o[kD];
#pragma unroll
  for (int d = 0; d < kD; ++d) o[d] = 0.0f;
  const float scale = rsqrtf(float(kD));
  const int last_q = min(q0 + kQ, tokens) - 1;
  const int seq = pos0 + last_q + 1;  // keys [0, seq) are needed by some row
  const int nblocks = (seq + kKeys - 1) / kKeys;
  const uint32_t lane_off = uint32_t(warp * 32) << 16;
  bool ok = true;

  for (int j = 0; j < nblocks && ok; ++j) {
    const int k0 = j * kKeys;
    // ---- stage K_j (rows = keys) and V_j^T (rows = dims, two 64-key halves)
    for (int i = threadIdx.x; i < kKeys * 8; i += kThreads) {
      const int r = i >> 3, c = (i & 7) * 8;
      uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
      if (k0 + r < seq) {
        kv = __ldcg(reinterpret_cast<const uint4*>(kb + size_t(k0 + r) * kD + c));
        vv = __ldcg(reinterpret_cast<const uint4*>(vb + size_t(k0 + r) * kD + c));
      }
      *reinterpret_cast<uint4*>(ks + sw(r, c)) = kv;
      // V^T: element (dim c+e, key r) -> sub-tile r / 64, row c+e, column r % 64
      const uint16_t* ve = reinterpret_cast<const uint16_t*>(&vv);
      unsigned char* vt = vs + (r >> 6) * (kD * 128);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        *reinterpret_cast<uint16_t*>(vt + sw(c + e, r & 63)) = ve[e];
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (threadIdx.x == 128) {
      // ---- S = Q K^T
      constexpr uint32_t idesc_s = idesc_bf16(128, kKeys);
#pragma unroll
      for (int kk = 0; kk < kD / 16; ++kk) {
        mma_bf16(tmem + kColS, desc_sw128(smem_u32(qs) + kk * 32),
                 desc_sw128(smem_u32(ks) + kk * 32), idesc_s, kk > 0 ? 1u : 0u);
      }
      mma_commit(bar_s);
    }
    if (warp < 4) {
      // ---- softmax of this block for query row `row`
      ok = __all_sync(0xffffffffu, wait_a(bar_s, uint32_t(j & 1), abort_flag));
      tc_fence_after();
      // pass 1: block maximum over the valid keys (S read 32 columns at a time)
      float mb = -FLT_MAX;
#pragma unroll 1
      for (int c0 = 0; c0 < kKeys; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_off + kColS + c0, r);
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          if (k0 + c0 + c <= qpos) mb = fmaxf(mb, __uint_as_float(r[c]) * scale);
        }
      }
      const float m_new = fmaxf(m_run, mb);
      const float alpha = m_run == -FLT_MAX ? 0.0f : __expf(m_run - m_new);
      // pass 2: P = exp(S - max) as BF16 into TMEM; the normaliser sums the
      // same BF16-rounded weights that P.V multiplies
      float lsum = 0.0f;
#pragma unroll 1
      for (int c0 = 0; c0 < kKeys; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_off + kColS + c0, r);
        uint32_t p[16];
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          const bool v0 = k0 + c0 + c <= qpos, v1 = k0 + c0 + c + 1 <= qpos;
          const float p0 = v0 ? __expf(__uint_as_float(r[c]) * scale - m_new) : 0.0f;
          const float p1 = v1 ? __expf(__uint_as_float(r[c + 1]) * scale - m_new) : 0.0f;
          const bf162 h = __floats2bfloat162_rn(p0, p1);
          lsum += __low2float(h) + __high2float(h);
          p[c / 2] = *reinterpret_cast<const uint32_t*>(&h);
        }
        tmem_st16(tmem + lane_off + kColP + c0 / 2, p);
      }
      l_run = l_run * alpha + lsum;
      m_run = m_new;
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar_p);
      // ---- O_j = P V, folded into the register accumulator
      ok = ok && __all_sync(0xffffffffu, wait_a(bar_o, uint32_t(j & 1), abort_flag));
      tc_fence_after();
#pragma unroll
      for (int c0 = 0; c0 < kD; c0 += 32) {
        uint32_t ov[32];
        tmem_ld32(tmem + lane_off + kColO + c0, ov);
#pragma unroll
        for (int d = 0; d < 32; ++d) o[c0 + d] = fmaf(o[c0 + d], alpha, __uint_as_float(ov[d]));
      }
    } else if (threadIdx.x == 128) {
      ok = wait_a(bar_p, uint32_t(j & 1), abort_flag);
      if (ok) {
        tc_fence_after();
        // P [128 x 128 keys] from TMEM (8 MMAs of K=16), V^T sub-tile per 64 keys
        constexpr uint32_t idesc_o = idesc_bf16(128, kD);
#pragma unroll
        for (int kk = 0; kk < kKeys / 16; ++kk) {
          mma_bf16_ta(tmem + kColO, tmem + kColP + kk * 8,
                      desc_sw128(smem_u32(vs) + (kk >> 2) * (kD * 128) + (kk & 3) * 32),
                      idesc_o, kk > 0 ? 1u : 0u);
        }
      }
      mma_commit(bar_o);
    }
    tc_fence_before();
    __syncthreads();  // K_j / V_j and the TMEM regions are free again
    tc_fence_after();
    ok = !*abort_flag;
  }

  if (warp < 4 && q0 + row < tokens && ok) {
    const float inv = l_run > 0.0f ? 1.0f / l_run : 0.0f;
    bf16* dst = out + size_t(q0 + row) * out_stride + head * kD;
#pragma unroll
    for (int d = 0; d < kD; d += 8) {
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const bf162 h = __floats2bfloat162_rn(o[d + 2 * e] * inv, o[d + 2 * e + 1] * inv);
        w[e] = *reinterpret_cast<const uint32_t*>(&h);
      }
      *reinterpret_cast<uint4*>(dst + d) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256)
                 : "memory");
  }
}

}  // namespace

cudaError_t launch_attention_prefill_tc(const bf16* q, int q_stride, const bf16* kcache,
                                        const bf16* vcache, bf16* out, int out_stride, int tokens,
                                        int pos0, int heads, int kv_heads, int max_seq,
                                        cudaStream_t stream) {
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(attention_prefill_tc_kernel,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(heads, (tokens + kQ - 1) / kQ);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, attention_prefill_tc_kernel, q, q_stride, kcache, vcache, out,
                            out_stride, tokens, pos0, heads, kv_heads, max_seq);
}

}  // namespace b200
