// GEMM activation preamble on the device: rotate (normalised FWHT in hsz
// blocks), quantise per row to symmetric int8, tile-pack for the GEMM.
//
// Reference: fgm_prep_rows (ops.c:293-314) = memcpy -> fgm_fwht (ops.c:153-175)
// -> fgm_quant_act (ops.c:181-204) -> pack (ops.c:302-313).
//
// One CTA per row.  The row is staged in shared memory; every FWHT stage is
// the reference's butterfly pairing (j, j + len) for len = 1, 2, 4, ...,
// computed as u + v and u - v with one rounding each, so the rotated values
// are bit-identical whatever thread computes them.  The normalisation
// multiply covers only the 16-wide chunks the reference's vector loop covers
// (ops.c:172), which leaves blocks smaller than 16 unscaled exactly as there.
// The scale is m / 127 and its inverse 1 / s with IEEE division, the
// quantised value rne(x * inv) with x86 saturation semantics.

#include "fgm_common.cuh"
#include "fgm_internal.h"

namespace fgm {

namespace {

constexpr int kPrepThreads = 256;

__device__ __forceinline__ float block_max(float v, float *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float u = __shfl_xor_sync(0xffffffffu, v, o);
    v = u > v ? u : v;
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float u = __shfl_xor_sync(0xffffffffu, v, o);
      v = u > v ? u : v;
    }
    if (lane == 0) red[0] = v;
  }
  __syncthreads();
  return red[0];
}

// grid.x covers rows [r0, rend) where rend is the end of the last 16-row tile
// block touched.  Rows < r1 are prepared; rows in [r1, rend) only fill their
// packed-tile rows: zeros past m, else a copy of qa (ops.c:306-311).
__global__ void __launch_bounds__(kPrepThreads) prep_kernel(const PrepParams p) {
  extern __shared__ float row[];
  __shared__ float red[32];
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // src comes from earlier kernels
  const int r = p.r0 + blockIdx.x;
  const int k = p.k, KB = k / kTileK;
  int8_t *pa_row = p.pa + ((size_t)(r / 16) * KB) * kATile + (size_t)(r % 16) * 64;

  if (r >= p.r1) {  // tile padding rows of the last block
    for (int i = threadIdx.x * 4; i < k; i += kPrepThreads * 4) {
      uint32_t v = 0;
      if (r < p.m) v = *reinterpret_cast<const uint32_t *>(p.qa + (size_t)r * k + i);
      *reinterpret_cast<uint32_t *>(pa_row + (size_t)(i / 64) * kATile + (i % 64)) = v;
    }
    return;
  }

  const float *src = p.src + (size_t)r * p.lda;
  for (int i = threadIdx.x; i < k; i += kPrepThreads) row[i] = src[i];

  if (p.hsz > 1) {
    const int hsz = p.hsz, half = hsz >> 1;
    for (int len = 1; len < hsz; len <<= 1) {
      __syncthreads();
      for (int q = threadIdx.x; q < (k >> 1); q += kPrepThreads) {
        const int blk = q / half, w = q % half;
        const int j = blk * hsz + (w / len) * (len << 1) + (w % len);
        const float u = row[j], v = row[j + len];
        row[j] = __fadd_rn(u, v);
        row[j + len] = __fsub_rn(u, v);
      }
    }
    __syncthreads();
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)hsz));
    const int scaled = hsz / 16 * 16;
    for (int i = threadIdx.x; i < k; i += kPrepThreads)
      if ((i % hsz) < scaled) row[i] = __fmul_rn(row[i], scale);
  }
  __syncthreads();
  if (p.rot)
    for (int i = threadIdx.x; i < k; i += kPrepThreads) p.rot[(size_t)r * k + i] = row[i];

  float m = 0.0f;
  for (int i = threadIdx.x; i < k; i += kPrepThreads) {
    const float a = fabsf(row[i]);
    m = a > m ? a : m;
  }
  m = block_max(m, red);
  const float s = (m == 0.0f) ? 1.0f : __fdiv_rn(m, 127.0f);
  const float inv = __fdiv_rn(1.0f, s);
  if (threadIdx.x == 0) p.qs[r] = s;

  for (int i = threadIdx.x * 4; i < k; i += kPrepThreads * 4) {
    uint32_t packed = 0;
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const int q = cvt_sat_i8(__fmul_rn(row[i + e], inv));
      packed |= (uint32_t)(q & 0xFF) << (8 * e);
    }
    if (p.qa) *reinterpret_cast<uint32_t *>(p.qa + (size_t)r * k + i) = packed;
    *reinterpret_cast<uint32_t *>(pa_row + (size_t)(i / 64) * kATile + (i % 64)) = packed;
  }
}

}  // namespace

size_t prep_smem_bytes(int k) { return (size_t)k * sizeof(float); }

cudaError_t launch_prep(const PrepParams &p, bool pdl, cudaStream_t st) {
  if (p.r0 >= p.r1) return cudaSuccess;
  const int rend = (p.r1 + 15) / 16 * 16;
  const size_t smem = prep_smem_bytes(p.k);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(rend - p.r0);
  cfg.blockDim = dim3(kPrepThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, prep_kernel, p);
}

}  // namespace fgm
