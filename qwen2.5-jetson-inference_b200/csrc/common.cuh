// Shared device helpers for the sm_100a Linear kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "b200_linear.h"

namespace b200 {

using bf16 = __nv_bfloat16;
using bf162 = __nv_bfloat162;

// BF16 bit pattern <-> float without going through the intrinsics' types.
__device__ __forceinline__ float bf16_lo(uint32_t pair) {
  return __uint_as_float(pair << 16);
}
__device__ __forceinline__ float bf16_hi(uint32_t pair) {
  return __uint_as_float(pair & 0xffff0000u);
}

// Exact int8 -> float for one byte of a packed word.
// Published magic-number method (the one FasterTransformer / CUTLASS use for
// fast integer-to-float conversion): XOR the byte with 0x80 to get u = q+128,
// place u in the low mantissa bits of 2^23 (0x4B000000), which is the float
// 8388608 + u exactly, then subtract 8388608 + 128.  Two ALU ops, no I2F.
template <int BYTE>
__device__ __forceinline__ float s8_to_f32_biased(uint32_t biased_word) {
  // biased_word = packed ^ 0x80808080
  constexpr uint32_t sel = 0x7540u | BYTE;  // bytes: [u_BYTE, 0, 0, 0x4B]
  return __uint_as_float(__byte_perm(biased_word, 0x4B000000u, sel)) -
         8388736.0f;
}

// Reads the global nanosecond timer (used to bound waits).
__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Programmatic dependent launch controls (no-ops when the launch carries no
// programmatic dependency).
__device__ __forceinline__ void pdl_wait_primary() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Orderable 32-bit key of a float: larger float -> larger unsigned key.
__device__ __forceinline__ uint32_t float_order_key(float v) {
  const uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

}  // namespace b200
