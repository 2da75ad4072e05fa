// Shared device helpers for the sm_100a kernels of the fgm-kernels GEMM path.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace fgm {

constexpr int kTileK = 64;      // K values per weight / activation tile
constexpr int kQ4Tile = 512;    // bytes of one int4 weight tile (16 n x 64 k)
constexpr int kQ8Tile = 1024;   // bytes of one int8 weight tile
constexpr int kATile = 1024;    // bytes of one packed activation tile (16 m x 64 k)

// Streamed-once weight word: bypass L1, the data is never re-read by this SM.
__device__ __forceinline__ uint32_t ld_stream_u32(const void *p) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// Activation word: re-read by every CTA, keep it in L1.
__device__ __forceinline__ uint32_t ld_shared_ro_u32(const void *p) {
  uint32_t v;
  asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// D += A(16x32 s8, row) * B(32x8 s8, col), int32 accumulate.
__device__ __forceinline__ void mma_s8_m16n8k32(int32_t (&d)[4], uint32_t a0, uint32_t a1,
                                                uint32_t a2, uint32_t a3, uint32_t b0,
                                                uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// D = A * B + C with separate C inputs (C may be a shared zero register).
__device__ __forceinline__ void mma_s8_m16n8k32_c(int32_t (&d)[4], uint32_t a0, uint32_t a1,
                                                  uint32_t a2, uint32_t a3, uint32_t b0,
                                                  uint32_t b1, int32_t c0, int32_t c1, int32_t c2,
                                                  int32_t c3) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};\n"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c0), "r"(c1), "r"(c2),
        "r"(c3));
}

// Two's-complement nibbles of a packed int4 word, each moved into the high
// half of its byte: byte i of the result is 16 * sext4(nibble).  Low nibbles
// (values 0..31 of a 64-value row) and high nibbles (values 32..63).
__device__ __forceinline__ uint32_t nib_lo_x16(uint32_t w) { return (w << 4) & 0xF0F0F0F0u; }
__device__ __forceinline__ uint32_t nib_hi_x16(uint32_t w) { return w & 0xF0F0F0F0u; }

// x86 _mm512_cvtps_epi32 + _mm512_cvtsepi32_epi8: round to nearest even,
// NaN or |v| >= 2^31 -> INT32_MIN, then signed saturation to int8.
__device__ __forceinline__ int cvt_sat_i8(float v) {
  int i;
  if (!(v >= -2147483648.0f && v < 2147483648.0f)) i = INT32_MIN;
  else i = __float2int_rn(v);
  return i > 127 ? 127 : (i < -128 ? -128 : i);
}

// The same pair as one saturating round-to-nearest-even conversion plus a
// select: NaN and |v| >= 2^31 (x86 INT32_MIN) give -128.  Returns the byte in
// the low 8 bits.
__device__ __forceinline__ uint32_t q8_x86(float v) {
  int i;
  asm("cvt.rni.sat.s8.f32 %0, %1;" : "=r"(i) : "f"(v));
  return fabsf(v) < 2147483648.0f ? (uint32_t)i : 0x80u;
}

// Four values scaled by inv and quantised, packed little-endian in a word.
__device__ __forceinline__ uint32_t q8_quad(float4 v, float inv) {
  const uint32_t a = q8_x86(__fmul_rn(v.x, inv)), b = q8_x86(__fmul_rn(v.y, inv));
  const uint32_t c = q8_x86(__fmul_rn(v.z, inv)), d = q8_x86(__fmul_rn(v.w, inv));
  return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

}  // namespace fgm
