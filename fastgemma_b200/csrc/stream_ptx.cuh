// Inline-PTX helpers shared by the weight-streaming decode kernels (gemv.cu,
// worklist.cu): bulk copies into shared memory, programmatic dependent
// launch, shared-memory loads, f16 scale words and the exact int32 -> f32
// group conversion.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

#include "tc_ptx.cuh"

namespace fgm {
namespace stream {

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes,
                                         uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(dst),
      "l"(src), "r"(bytes), "r"(tc::smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ uint32_t lds32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}

__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(a));
  return v;
}

__device__ __forceinline__ uint32_t ldg_stream_u32(const void *p) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ float f16_to_f32(uint32_t bits16) {
  return __half2float(__ushort_as_half((unsigned short)bits16));
}

// The scale pair (columns g and g+8 of a group row) of thread (g, .), from the
// 8-word row held one word per lane at lanes base..base+7 of register v.
__device__ __forceinline__ void scale_pair(uint32_t v, int base, int g8, float &s0, float &s1) {
  const uint32_t w0 = __shfl_sync(0xffffffffu, v, base + (g8 >> 1));
  const uint32_t w1 = __shfl_sync(0xffffffffu, v, base + 4 + (g8 >> 1));
  const int sh = (g8 & 1) * 16;
  s0 = f16_to_f32(w0 >> sh);
  s1 = f16_to_f32(w1 >> sh);
}

// Exact int32 -> f32 for |x| <= 2^22 without the quarter-rate converter:
// 1.5 * 2^23 + x is an exact float whose mantissa holds x, so subtracting
// 1.5 * 2^23 recovers x.  A scale group's sum fits when the group has at
// most 4096 values (|a * w| <= 128 * 8 per product); larger groups convert
// with cvt (i2f_group).
constexpr int kExactGroupMax = 4096;
__device__ __forceinline__ float i2f_exact(int32_t x) {
  return __fadd_rn(__int_as_float(x + 0x4B400000), -12582912.0f);
}
__device__ __forceinline__ float i2f_group(int32_t x, bool exact_ok) {
  return exact_ok ? i2f_exact(x) : __int2float_rn(x);
}

}  // namespace stream
}  // namespace fgm
