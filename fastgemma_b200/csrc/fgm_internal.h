// Internal launch interfaces between the C ABI (fgm_cuda.cu) and the kernels.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace fgm {

struct GemvParams {
  int M, N, K, group;       // group: int4 scale group; unused for int8
  const int8_t *A;          // packed activations [ceil(M/16)][K/64][16][64]
  const float *a_scale;     // [M]
  const uint8_t *B;         // weight tiles (int4 nibbles or int8), as bytes
  const void *b_scale;      // f16 [K/group][N] (int4) or f32 [N] (int8)
  float *C;                 // output, element (m, n) at C[m*ldc + n - c_col0]
  int ldc;
  int c_col0;
  int32_t *acc;             // raw accumulator output (debug launches)
  int nb0;                  // first n-block of the range
  int *err;                 // device flag set when a bounded wait gives up (may be null)
};

// Launch geometry of the streaming decode kernel (gemv.cu).
struct GemvPlan {
  int warps;        // warps per CTA
  int parts;        // warps sharing one n-block (split K), a power of two
  int units;        // n-blocks in the range
  int chunk_tiles;  // weight tiles per ring stage
  int stages;       // ring depth per warp
  int stage_bytes;
  int xchg_bytes;   // per-team exchange area for split K
  int a_bytes;      // activations staged in shared memory (0: read from global)
  int ctas_per_sm;  // resident CTAs per SM the shared-memory budget allows
  int grid_x;
  size_t smem_bytes;
};

GemvPlan plan_gemv(const GemvParams &p, int nblocks, bool q4, int num_sms, size_t smem_limit);

// nblocks n-blocks starting at p.nb0; q4 selects the int4 layout; a non-null
// p.acc writes int32 accumulators instead of the f32 epilogue; pdl launches
// with programmatic stream serialisation (weight prefetch overlaps the
// previous kernel).
cudaError_t launch_gemv(const GemvParams &p, int nblocks, bool q4, bool pdl, int num_sms,
                        size_t smem_limit, cudaStream_t st);

struct PrepParams {
  const float *src;
  int lda;
  float *rot;    // may be null
  int8_t *qa;    // may be null
  float *qs;
  int8_t *pa;
  int m, k, hsz, r0, r1;
};

cudaError_t launch_prep(const PrepParams &p, bool pdl, cudaStream_t st);

// Number of kernel launches issued by this library (instrumentation).
void count_launch(int n = 1);

}  // namespace fgm
