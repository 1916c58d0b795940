// Causal GQA attention of one query row against a BF16 KV cache (head_dim
// 64), shared by the engine's standalone attention kernel (prefill and the
// graph decode step) and by the persistent decode kernel.
//
// Arithmetic (reference src/cuda/kernels.cu:159-283): FP32 scores
// q.k / sqrt(64) over BF16 q and k, FP32 softmax with the row maximum
// subtracted, FP32 weighted sum of BF16 v, output rounded to BF16 once.
//
// Work split over NT threads (NT / 32 warps):
//   scores:  one position per thread (a 128-byte K row read as 8 x 16 B);
//   softmax: block max and block sum through shared memory;
//   P.V:     one position per warp at a time, lane l owning dims 2l, 2l+1
//            (a warp reads one coalesced 128-byte V row), per-warp partial
//            sums added across warps at the end.
#pragma once

#include <cfloat>

#include "common.cuh"

namespace b200 {

constexpr int kHeadDim = 64;

// Shared-memory scratch of attend_row: scores[seq_cap] + red[NT/32] +
// part[NT/32][64] floats.
template <int NT>
__host__ __device__ constexpr size_t attend_smem_floats(int seq_cap) {
  return size_t(seq_cap) + NT / 32 + size_t(NT / 32) * kHeadDim;
}

// q: 64 FP32 values in shared memory.  kbase / vbase: this KV head's cache
// rows [pos][64].  Positions [0, seq) are attended; position `cur` (or -1)
// is taken from kcur / vcur (64 FP32 values in shared memory) instead of
// the cache.  `sync()` synchronises the NT threads.  Thread `tid` < 64
// calls store(tid, output value of dimension tid).
template <int NT, class Sync, class Store>
__device__ __forceinline__ void attend_row(const float* qs, const bf16* kbase,
                                           const bf16* vbase, int seq, int cur,
                                           const float* kcur, const float* vcur,
                                           float* smem, int tid, Sync sync,
                                           Store store) {
  constexpr int NW = NT / 32;
  float* scores = smem;
  float* red = smem + seq;
  float* part = red + NW;
  const int lane = tid & 31, warp = tid >> 5;
  const float scale = rsqrtf(float(kHeadDim));
  float mx = -FLT_MAX;
  for (int p = tid; p < seq; p += NT) {
    float dot = 0.0f;
    if (p == cur) {
#pragma unroll 16
      for (int d = 0; d < kHeadDim; ++d) dot = fmaf(qs[d], kcur[d], dot);
    } else {
      const uint4* kr = reinterpret_cast<const uint4*>(kbase + size_t(p) * kHeadDim);
      uint4 w[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) w[c] = __ldcg(kr + c);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        dot = fmaf(qs[8 * c + 0], bf16_lo(w[c].x), dot);
        dot = fmaf(qs[8 * c + 1], bf16_hi(w[c].x), dot);
        dot = fmaf(qs[8 * c + 2], bf16_lo(w[c].y), dot);
        dot = fmaf(qs[8 * c + 3], bf16_hi(w[c].y), dot);
        dot = fmaf(qs[8 * c + 4], bf16_lo(w[c].z), dot);
        dot = fmaf(qs[8 * c + 5], bf16_hi(w[c].z), dot);
        dot = fmaf(qs[8 * c + 6], bf16_lo(w[c].w), dot);
        dot = fmaf(qs[8 * c + 7], bf16_hi(w[c].w), dot);
      }
    }
    const float s = dot * scale;
    scores[p] = s;
    mx = fmaxf(mx, s);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  if (lane == 0) red[warp] = mx;
  sync();
  mx = red[0];
#pragma unroll
  for (int w = 1; w < NW; ++w) mx = fmaxf(mx, red[w]);
  sync();
  float sum = 0.0f;
  for (int p = tid; p < seq; p += NT) {
    const float e = expf(scores[p] - mx);
    scores[p] = e;
    sum += e;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
  if (lane == 0) red[warp] = sum;
  sync();  // scores[] complete, red[] holds the partial sums
  float a0 = 0.0f, a1 = 0.0f;
  const uint32_t* vrow = reinterpret_cast<const uint32_t*>(vbase) + lane;
  int p = warp;
  for (; p + 3 * NW < seq; p += 4 * NW) {
    uint32_t v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int q = p + j * NW;
      v[j] = q == cur ? 0u : __ldcg(vrow + size_t(q) * (kHeadDim / 2));
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int q = p + j * NW;
      const float pr = scores[q];
      const float v0 = q == cur ? vcur[2 * lane] : bf16_lo(v[j]);
      const float v1 = q == cur ? vcur[2 * lane + 1] : bf16_hi(v[j]);
      a0 = fmaf(pr, v0, a0);
      a1 = fmaf(pr, v1, a1);
    }
  }
  for (; p < seq; p += NW) {
    const float pr = scores[p];
    float v0, v1;
    if (p == cur) {
      v0 = vcur[2 * lane];
      v1 = vcur[2 * lane + 1];
    } else {
      const uint32_t v = __ldcg(vrow + size_t(p) * (kHeadDim / 2));
      v0 = bf16_lo(v);
      v1 = bf16_hi(v);
    }
    a0 = fmaf(pr, v0, a0);
    a1 = fmaf(pr, v1, a1);
  }
  part[warp * kHeadDim + 2 * lane] = a0;
  part[warp * kHeadDim + 2 * lane + 1] = a1;
  sync();
  if (tid < kHeadDim) {
    float denom = 0.0f, o = 0.0f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      denom += red[w];
      o += part[w * kHeadDim + tid];
    }
    store(tid, o / denom);
  }
  sync();  // smem reusable by the caller
}

}  // namespace b200
