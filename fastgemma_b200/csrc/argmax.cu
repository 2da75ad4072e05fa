// Row argmax of logits, split over column ranges and ranks, with the
// reference's semantics (fgm-serve/src/engine.rs:75-83, fgm-bench
// src/main.rs:201-209): scan columns in ascending order keeping the first
// strictly greater value, starting from (0, -inf) -- so NaN never wins, ties
// keep the lowest index, and a row with no value above -inf answers 0.
//
// A partial result is (value, index) with index -1 meaning "nothing above
// -inf".  Partials merge associatively: the larger value wins, equal values
// keep the lower index; so per-chunk, per-rank partials merged in any order
// give the sequential scan's answer.

#include "fgm_common.cuh"
#include "fgm_internal.h"

namespace fgm {

namespace {

constexpr int kArgThreads = 256;

__device__ __forceinline__ void merge_pair(float &v, int &i, float v2, int i2) {
  if (i2 < 0) return;
  if (i < 0 || v2 > v || (v2 == v && i2 < i)) {
    v = v2;
    i = i2;
  }
}

__device__ __forceinline__ void block_merge(float &v, int &i, float *sv, int *si) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, i, o);
    merge_pair(v, i, v2, i2);
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    sv[warp] = v;
    si[warp] = i;
  }
  __syncthreads();
  if (warp == 0) {
    v = lane < (int)(blockDim.x >> 5) ? sv[lane] : 0.0f;
    i = lane < (int)(blockDim.x >> 5) ? si[lane] : -1;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
      const int i2 = __shfl_xor_sync(0xffffffffu, i, o);
      merge_pair(v, i, v2, i2);
    }
  }
}

// grid (chunks, M): chunk c of row m -> part[m][c]; indices are col0 + column.
__global__ void __launch_bounds__(kArgThreads) argmax_chunks(const float *__restrict__ C, int N,
                                                             int ldc, int col0, int chunk,
                                                             float *pv, int *pi) {
  __shared__ float sv[kArgThreads / 32];
  __shared__ int si[kArgThreads / 32];
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // logits come from earlier kernels
  const int m = blockIdx.y, c0 = blockIdx.x * chunk, c1 = min(N, c0 + chunk);
  const float *row = C + (size_t)m * ldc;
  float v = -INFINITY;
  int i = -1;
  for (int n = c0 + threadIdx.x; n < c1; n += kArgThreads) {
    const float x = row[n];
    if (x > v) {  // strictly greater: NaN and -inf never enter
      v = x;
      i = col0 + n;
    }
  }
  block_merge(v, i, sv, si);
  if (threadIdx.x == 0) {
    pv[(size_t)m * gridDim.x + blockIdx.x] = v;
    pi[(size_t)m * gridDim.x + blockIdx.x] = i;
  }
}

// One warp per row: merge P partials per row (row m's partials at stride 1
// from m*P), answer 0 where nothing was above -inf.
__global__ void argmax_merge(const float *__restrict__ pv, const int *__restrict__ pi, int M,
                             int P, int *out) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int lane = threadIdx.x & 31;
  const int m = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (m >= M) return;
  float v = -INFINITY;
  int i = -1;
  for (int p = lane; p < P; p += 32) merge_pair(v, i, pv[(size_t)m * P + p], pi[(size_t)m * P + p]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, i, o);
    merge_pair(v, i, v2, i2);
  }
  if (lane == 0) out[m] = i < 0 ? 0 : i;
}

cudaError_t pdl_launch(cudaLaunchConfig_t &cfg, bool pdl, cudaLaunchAttribute *attr) {
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaSuccess;
}

}  // namespace

int argmax_chunk_count(int N) { return (N + kArgmaxChunk - 1) / kArgmaxChunk; }

cudaError_t launch_argmax_partials(const float *C, int M, int N, int ldc, int col0, float *pv,
                                   int *pi, bool pdl, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(argmax_chunk_count(N), M);
  cfg.blockDim = dim3(kArgThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  pdl_launch(cfg, pdl, attr);
  return cudaLaunchKernelEx(&cfg, argmax_chunks, C, N, ldc, col0, (int)kArgmaxChunk, pv, pi);
}

cudaError_t launch_argmax_merge(const float *pv, const int *pi, int M, int P, int *out, bool pdl,
                                cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((M + 7) / 8);
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  pdl_launch(cfg, pdl, attr);
  return cudaLaunchKernelEx(&cfg, argmax_merge, pv, pi, M, P, out);
}

}  // namespace fgm
