// GEMM activation preamble on the device: rotate (normalised FWHT in hsz
// blocks), quantise per row to symmetric int8, tile-pack for the GEMM.
//
// Reference: fgm_prep_rows (ops.c:293-314) = memcpy -> fgm_fwht (ops.c:153-175)
// -> fgm_quant_act (ops.c:181-204) -> pack (ops.c:302-313).
//
// prep_fast_kernel (hsz <= 1024, k <= 16384) keeps each row in registers, one
// warp per 1024 values.  prep_kernel covers the rest: one CTA per row.  The
// row is staged in shared memory; every FWHT stage is
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
      if (p.pa) *reinterpret_cast<uint32_t *>(pa_row + (size_t)(i / 64) * kATile + (i % 64)) = v;
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
    if (p.pa) *reinterpret_cast<uint32_t *>(pa_row + (size_t)(i / 64) * kATile + (i % 64)) = packed;
  }
}

// ------------------------------------------------------ register-resident
// For hsz <= 1024 and k <= 16384: one CTA per row, one warp per segment of
// 1024 values.  Lane l holds values 4l + 128j (j = 0..7) of its segment as
// v[j], so the float4 loads and stores are coalesced; FWHT strides 1 and 2
// pair float4 components, 4..64 pair lanes (shuffles), 128..512 pair
// registers.  Every butterfly output is the reference's u + v or u - v of
// the same operands, so the result equals the shared-memory version.
constexpr int kSeg = 1024;
constexpr int kSegV = kSeg / 128;
constexpr int kFastMaxK = 16 * kSeg;

__device__ __forceinline__ float4 f4_add(float4 a, float4 b) {
  return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z),
                     __fadd_rn(a.w, b.w));
}
__device__ __forceinline__ float4 f4_sub(float4 a, float4 b) {
  return make_float4(__fsub_rn(a.x, b.x), __fsub_rn(a.y, b.y), __fsub_rn(a.z, b.z),
                     __fsub_rn(a.w, b.w));
}

template <int JL>  // stride 128 * JL: registers j and j + JL
__device__ __forceinline__ void reg_pairs(float4 (&v)[kSegV]) {
#pragma unroll
  for (int j = 0; j < kSegV; j++) {
    if (j & JL) continue;
    const float4 u = v[j], w = v[j + JL];
    v[j] = f4_add(u, w);
    v[j + JL] = f4_sub(u, w);
  }
}

__device__ __forceinline__ float bfly_lane(float own, int lm, bool hi) {
  const float other = __shfl_xor_sync(0xffffffffu, own, lm);
  return hi ? __fsub_rn(other, own) : __fadd_rn(own, other);
}

__device__ __forceinline__ void fwht_seg(float4 (&v)[kSegV], int hsz, int lane) {
  for (int len = 1; len < hsz; len <<= 1) {
    if (len == 1) {
#pragma unroll
      for (int j = 0; j < kSegV; j++) {
        const float4 u = v[j];
        v[j] = make_float4(__fadd_rn(u.x, u.y), __fsub_rn(u.x, u.y), __fadd_rn(u.z, u.w),
                           __fsub_rn(u.z, u.w));
      }
    } else if (len == 2) {
#pragma unroll
      for (int j = 0; j < kSegV; j++) {
        const float4 u = v[j];
        v[j] = make_float4(__fadd_rn(u.x, u.z), __fadd_rn(u.y, u.w), __fsub_rn(u.x, u.z),
                           __fsub_rn(u.y, u.w));
      }
    } else if (len < 128) {
      const int lm = len >> 2;
      const bool hi = (lane & lm) != 0;
#pragma unroll
      for (int j = 0; j < kSegV; j++) {
        v[j].x = bfly_lane(v[j].x, lm, hi);
        v[j].y = bfly_lane(v[j].y, lm, hi);
        v[j].z = bfly_lane(v[j].z, lm, hi);
        v[j].w = bfly_lane(v[j].w, lm, hi);
      }
    } else if (len == 128) {
      reg_pairs<1>(v);
    } else if (len == 256) {
      reg_pairs<2>(v);
    } else {
      reg_pairs<4>(v);
    }
  }
}

__global__ void __launch_bounds__(512, 1) prep_fast_kernel(const PrepParams p) {
  __shared__ float red[16];
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // src comes from earlier kernels
  const int r = p.r0 + blockIdx.x;
  const int k = p.k, KB = k / kTileK;
  int8_t *pa_row = p.pa + ((size_t)(r / 16) * KB) * kATile + (size_t)(r % 16) * 64;
  if (r >= p.r1) {  // tile padding rows of the last block: zeros past m, else qa
    for (int i = threadIdx.x * 4; i < k; i += blockDim.x * 4) {
      uint32_t v = 0;
      if (r < p.m) v = *reinterpret_cast<const uint32_t *>(p.qa + (size_t)r * k + i);
      if (p.pa) *reinterpret_cast<uint32_t *>(pa_row + (size_t)(i / 64) * kATile + (i % 64)) = v;
    }
    return;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int seg0 = warp * kSeg, segn = min(kSeg, k - seg0);
  const float *src = p.src + (size_t)r * p.lda + seg0;
  const bool vec = ((reinterpret_cast<uintptr_t>(p.src) & 15) == 0) && (p.lda % 4 == 0);
  float4 v[kSegV];
#pragma unroll
  for (int j = 0; j < kSegV; j++) {
    const int e = j * 128 + lane * 4;
    if (e >= segn) {
      v[j] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    } else if (vec) {
      v[j] = *reinterpret_cast<const float4 *>(src + e);
    } else {
      v[j] = make_float4(src[e], src[e + 1], src[e + 2], src[e + 3]);
    }
  }
  if (p.hsz > 1) {
    fwht_seg(v, p.hsz, lane);
    if (p.hsz >= 16) {  // ops.c:172 scales the 16-wide chunks of each block
      const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)p.hsz));
#pragma unroll
      for (int j = 0; j < kSegV; j++) {
        v[j].x = __fmul_rn(v[j].x, scale);
        v[j].y = __fmul_rn(v[j].y, scale);
        v[j].z = __fmul_rn(v[j].z, scale);
        v[j].w = __fmul_rn(v[j].w, scale);
      }
    }
  }
  float mx = 0.0f;
#pragma unroll
  for (int j = 0; j < kSegV; j++) {
    const float a0 = fabsf(v[j].x), a1 = fabsf(v[j].y), a2 = fabsf(v[j].z), a3 = fabsf(v[j].w);
    mx = a0 > mx ? a0 : mx;
    mx = a1 > mx ? a1 : mx;
    mx = a2 > mx ? a2 : mx;
    mx = a3 > mx ? a3 : mx;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float u = __shfl_xor_sync(0xffffffffu, mx, o);
    mx = u > mx ? u : mx;
  }
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  mx = 0.0f;
  for (int w = 0; w < nw; w++) mx = red[w] > mx ? red[w] : mx;
  const float s = (mx == 0.0f) ? 1.0f : __fdiv_rn(mx, 127.0f);
  const float inv = __fdiv_rn(1.0f, s);
  if (threadIdx.x == 0) p.qs[r] = s;
#pragma unroll
  for (int j = 0; j < kSegV; j++) {
    const int e = j * 128 + lane * 4;
    if (e >= segn) continue;
    const int kk = seg0 + e;
    if (p.rot) *reinterpret_cast<float4 *>(p.rot + (size_t)r * k + kk) = v[j];
    const uint32_t w = q8_quad(v[j], inv);
    if (p.qa) *reinterpret_cast<uint32_t *>(p.qa + (size_t)r * k + kk) = w;
    if (p.pa) *reinterpret_cast<uint32_t *>(pa_row + (size_t)(kk / 64) * kATile + (kk % 64)) = w;
  }
}

// Two host-resident byte regions (page-locked, read through their device
// mapping) copied into device memory by one small kernel: the packed
// activations and their scales of a host-pointer GEMM call, without a
// copy-engine round trip each.  Word copies when both ends are 4-byte
// aligned, byte copies otherwise.
__global__ void pull_kernel(const uint8_t *s1, uint8_t *d1, size_t n1, const uint8_t *s2,
                            uint8_t *d2, size_t n2) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the buffers' earlier readers are done
  const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (int r = 0; r < 2; r++) {
    const uint8_t *s = r ? s2 : s1;
    uint8_t *d = r ? d2 : d1;
    const size_t n = r ? n2 : n1;
    if (!n) continue;
    if ((((uintptr_t)s | (uintptr_t)d | n) & 3) == 0) {
      const uint32_t *sw = reinterpret_cast<const uint32_t *>(s);
      uint32_t *dw = reinterpret_cast<uint32_t *>(d);
      for (size_t i = tid; i < n / 4; i += stride) dw[i] = sw[i];
    } else {
      for (size_t i = tid; i < n; i += stride) d[i] = s[i];
    }
  }
}

}  // namespace

cudaError_t launch_pull(const void *s1, void *d1, size_t n1, const void *s2, void *d2, size_t n2,
                        bool pdl, cudaStream_t st) {
  const size_t words = (n1 > n2 ? n1 : n2) / 4 + 1;
  unsigned blocks = (unsigned)((words + 255) / 256);
  if (blocks > 64) blocks = 64;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks);
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, pull_kernel, static_cast<const uint8_t *>(s1),
                            static_cast<uint8_t *>(d1), n1, static_cast<const uint8_t *>(s2),
                            static_cast<uint8_t *>(d2), n2);
}

size_t prep_smem_bytes(int k) { return (size_t)k * sizeof(float); }

cudaError_t launch_prep(const PrepParams &p, bool pdl, cudaStream_t st) {
  if (p.r0 >= p.r1) return cudaSuccess;
  const int rend = (p.r1 + 15) / 16 * 16;
  if (p.hsz <= kSeg && p.k <= kFastMaxK) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(rend - p.r0);
    cfg.blockDim = dim3((p.k + kSeg - 1) / kSeg * 32);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, prep_fast_kernel, p);
  }
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
