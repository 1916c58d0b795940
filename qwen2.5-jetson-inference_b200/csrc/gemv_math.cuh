// Dot-product and argmax helpers shared by the decode GEMV kernels
// (gemv.cu) and the persistent decode kernel (decode_persistent.cu).
#pragma once

#include <cfloat>
#include <climits>

#include "common.cuh"

namespace b200 {

// Strictly-greater update with lowest index on ties; values <= -FLT_MAX
// never win (reference argmax semantics, src/cuda/kernels.cu:326-356).
__device__ __forceinline__ void argmax_update(float& best, int& best_index,
                                              float v, int index) {
  if (v > best || (v == best && v > -FLT_MAX && index < best_index)) {
    best = v;
    best_index = index;
  }
}

__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }

// Packed: a += q(4 int8 of `packed`) * x[0..3].
__device__ __forceinline__ float2 dot4_s8_x2(uint32_t packed, float4 x,
                                             float2 a) {
  const uint32_t b = packed ^ 0x80808080u;
  const float2 bias = f2(-8388736.0f, -8388736.0f);
  const float2 q01 = __fadd2_rn(
      f2(__uint_as_float(__byte_perm(b, 0x4B000000u, 0x7540u)),
         __uint_as_float(__byte_perm(b, 0x4B000000u, 0x7541u))),
      bias);
  const float2 q23 = __fadd2_rn(
      f2(__uint_as_float(__byte_perm(b, 0x4B000000u, 0x7542u)),
         __uint_as_float(__byte_perm(b, 0x4B000000u, 0x7543u))),
      bias);
  a = __ffma2_rn(q01, f2(x.x, x.y), a);
  a = __ffma2_rn(q23, f2(x.z, x.w), a);
  return a;
}

__device__ __forceinline__ float2 dot4_bf16_x2(uint32_t w01, uint32_t w23,
                                               float4 x, float2 a) {
  a = __ffma2_rn(f2(bf16_lo(w01), bf16_hi(w01)), f2(x.x, x.y), a);
  a = __ffma2_rn(f2(bf16_lo(w23), bf16_hi(w23)), f2(x.z, x.w), a);
  return a;
}

}  // namespace b200
