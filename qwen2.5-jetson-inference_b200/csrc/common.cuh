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

__device__ __forceinline__ float bf16_round(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
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

// Upper bound of every spin-wait in the library (a healthy wait is
// microseconds; the bound only ends a wait that can no longer complete).
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;  // 2 s

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

// ------------------------------------------------------------ PTX wrappers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar,
                                                      uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
                   bar),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* tmap,
                                            int c0, int c1, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::"
      "complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(tmap), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 1-D bulk copy global -> shared (TMA engine), completes on an mbarrier.
// Addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src,
                                          uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// Bounded wait on the mbarrier phase with the given parity.  On expiry the
// error code is recorded in *status (first error wins), the CTA-wide abort
// flag is raised and false is returned; a raised flag also ends the wait.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar,
                                                  uint32_t parity,
                                                  volatile int* abort_flag,
                                                  int error_code,
                                                  int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (global_timer_ns() - start > kWaitTimeoutNs) {
      *abort_flag = 1;
      atomicCAS(status, 0, error_code);
      return false;
    }
  }
}

}  // namespace b200
