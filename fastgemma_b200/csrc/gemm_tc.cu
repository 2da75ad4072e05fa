// Prefill-shaped int8 GEMM on the 5th-generation tensor cores (tcgen05,
// kind::i8, int32 accumulators in tensor memory), fed by TMA.
//
// Reference: fgm_gemm_q8c (amx_gemm.c:444-475, 2x2 tile path INNER_Q8_2x2
// :375-410) and fgm_gemm_q8c_vnni (vnni_gemm.c:224-245):
//   C[m, n] = (float)(sum_k A[m,k] * W[n,k]) * (b_scale[n] * a_scale[m]).
//
// Operand layouts
// ---------------
// Both operands are K-major row-major byte matrices read through 2-D TMA
// boxes of 128-byte rows with the 128-byte swizzle, the canonical SW128
// K-major layout the MMA descriptors describe (8-row atoms of 1 KB).  The
// activations are the quantiser's row-major int8 output (fgm_quant_act's q,
// ops.c:181-204) or, for callers holding the tile-packed form (ops.c:279-290),
// a row-major copy of it.  The .fgm int8 weight tile [k/4][n][k%4]
// (convert/quant.py:96-107) is neither K- nor MN-major canonical, so a weight
// is prepared once into a row-major [N][K] copy.
//
// Pipeline
// --------
// One CTA owns a 256 x 128 output tile (two M=128 halves sharing each B
// tile) and walks K in 128-byte stages through a 4-deep ring: warp 0 (one
// lane) issues the TMA loads, warp 1 (one lane) issues four K=32 MMAs per
// half per stage and commits each stage back to the producer, warp 2 owns
// the tensor-memory allocation, warps 4-7 drain the accumulators (tcgen05.ld,
// 32 lanes each) and apply the f32 epilogue.  Every mbarrier wait is bounded
// in time; a kernel that gives up sets the device error flag and still
// releases its tensor memory.

#include <cuda.h>

#include <cstring>

#include "fgm_common.cuh"
#include "fgm_internal.h"
#include "tc_ptx.cuh"

namespace fgm {

namespace {

constexpr int kTcBM = 256;  // two M=128 halves
constexpr int kTcBN = 128;
constexpr int kTcBK = 128;  // bytes of K per stage
constexpr int kTcThreads = 256;
constexpr int kTcA = kTcBM * kTcBK;
constexpr int kTcB = kTcBN * kTcBK;
constexpr int kTcStage = kTcA + kTcB;
constexpr int kTcTmemCols = 2 * kTcBN;

__device__ __forceinline__ void st_global_v4(float *p, float a, float b, float c, float d) {
  asm volatile("st.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

__global__ void __launch_bounds__(kTcThreads, 1)
    q8c_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                  const __grid_constant__ CUtensorMap tmC, const TcParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // stage buffers must sit on 1 KB boundaries for the swizzle pattern
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int S = p.stages;
  constexpr size_t kOutBytes = (size_t)(kTcBN / 32) * kTcBM * 128;  // staged f32 tile
  const size_t ring = (size_t)S * kTcStage > kOutBytes ? (size_t)S * kTcStage : kOutBytes;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + ring);
  uint64_t *empty = full + S;
  uint64_t *accum = empty + S;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accum + 1);
  __shared__ int s_fail;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KS = (p.K + kTcBK - 1) / kTcBK;
  const int m0 = blockIdx.y * kTcBM;
  const int n0 = p.nb0 * 16 + blockIdx.x * kTcBN;

  if (threadIdx.x == 0) {
    s_fail = 0;
    for (int s = 0; s < S; s++) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    tc::mbar_init(accum, 1);
    tc::fence_mbar_init();
    tc::prefetch_tmap(&tmA);
    tc::prefetch_tmap(&tmB);
  }
  if (warp == 2) {
    tc::tmem_alloc(tmem_slot, kTcTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == 0 && lane == 0) {  // ---------------------------------- producer
    asm volatile("griddepcontrol.wait;" ::: "memory");  // activations from earlier kernels
    for (int ks = 0; ks < KS; ks++) {
      const int s = ks % S;
      if (ks >= S && !tc::mbar_wait(&empty[s], ((ks / S) & 1) ^ 1)) {
        s_fail = 1;
        break;
      }
      uint8_t *sa = smem + (size_t)s * kTcStage;
      tc::mbar_expect_tx(&full[s], kTcStage);
      tc::tma_load_2d(sa, &tmA, &full[s], ks * kTcBK, m0);
      tc::tma_load_2d(sa + kTcA, &tmB, &full[s], ks * kTcBK, n0);
    }
  } else if (warp == 1 && lane == 0) {  // ---------------------------- MMA
    const uint32_t idesc = tc::idesc_i8(128, kTcBN);
    for (int ks = 0; ks < KS; ks++) {
      const int s = ks % S;
      if (!tc::mbar_wait(&full[s], (ks / S) & 1)) {
        s_fail = 1;
        break;
      }
      tc::fence_after_sync();
      const uint32_t sa = tc::smem_u32(smem + (size_t)s * kTcStage);
      const uint32_t sb = sa + kTcA;
#pragma unroll
      for (int h = 0; h < 2; h++)
#pragma unroll
        for (int j = 0; j < kTcBK / 32; j++)  // K=32 slices of the 128-byte stage
          tc::mma_i8(tmem + h * kTcBN, tc::sdesc_sw128(sa + h * 128 * kTcBK + j * 32),
                     tc::sdesc_sw128(sb + j * 32), idesc, (ks | j) != 0);
      tc::mma_commit(&empty[s]);  // stage s is free once these MMAs complete
    }
    tc::mma_commit(accum);
  } else if (warp >= 4) {  // ------------------------------------- epilogue
    const int q = warp - 4;  // TMEM lane quadrant
    bool ok = tc::mbar_wait(accum, 0);
    if (!ok) s_fail = 1;
    tc::fence_after_sync();
    if (ok) {
      asm volatile("griddepcontrol.wait;" ::: "memory");
      // f32 tile staged in the (now idle) ring as four 32-column blocks of
      // [256 rows][128 B], 128-byte swizzled, then written by TMA stores that
      // the output map clips to rows < M and columns [nb0*16, n_end).
      const bool tma_out = p.tma_store && !p.acc;
#pragma unroll 1
      for (int h = 0; h < 2; h++) {
        const int ml = h * 128 + q * 32 + lane;
        const int m = m0 + ml;
        const bool row_ok = m < p.M;
        const float as = (row_ok && p.a_scale) ? p.a_scale[m] : 0.0f;
        // 64 columns per round: two 32-column TMEM loads in flight, one wait
#pragma unroll 1
        for (int c64 = 0; c64 < kTcBN / 64; c64++) {
          uint32_t v[64];
          const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + h * kTcBN + c64 * 64;
          tc::tmem_ld_x32(ta, v);
          tc::tmem_ld_x32(ta + 32, v + 32);
          tc::tmem_wait_ld();
#pragma unroll
          for (int cc = 0; cc < 4; cc++) {
            const int c = c64 * 4 + cc;  // 16-column chunk of the tile
            const int n = n0 + c * 16;
            if (p.acc) {
              if (row_ok && n < p.n_end)
                for (int e = 0; e < 16; e++)
                  p.acc[(size_t)m * p.N + n + e] = (int32_t)v[cc * 16 + e];
              continue;
            }
            if (n >= p.n_end) continue;
            float o[16];
            const float4 *bs4 = reinterpret_cast<const float4 *>(p.b_scale + n);
#pragma unroll
            for (int e4 = 0; e4 < 4; e4++) {
              const float4 b = __ldg(bs4 + e4);
              const uint32_t *u = v + cc * 16 + 4 * e4;
              o[4 * e4 + 0] = __fmul_rn(__int2float_rn((int32_t)u[0]), __fmul_rn(b.x, as));
              o[4 * e4 + 1] = __fmul_rn(__int2float_rn((int32_t)u[1]), __fmul_rn(b.y, as));
              o[4 * e4 + 2] = __fmul_rn(__int2float_rn((int32_t)u[2]), __fmul_rn(b.z, as));
              o[4 * e4 + 3] = __fmul_rn(__int2float_rn((int32_t)u[3]), __fmul_rn(b.w, as));
            }
            if (tma_out) {
              uint8_t *rowp = smem + (size_t)(c >> 1) * (kTcBM * 128) + (size_t)ml * 128;
#pragma unroll
              for (int t = 0; t < 4; t++) {
                const int j = (c & 1) * 4 + t;  // 16-byte chunk inside the 128-byte row
                *reinterpret_cast<float4 *>(rowp + ((j ^ (ml & 7)) << 4)) =
                    make_float4(o[4 * t], o[4 * t + 1], o[4 * t + 2], o[4 * t + 3]);
              }
            } else if (row_ok) {
              float *dst = p.C + (size_t)m * p.ldc + (n - p.c_col0);
#pragma unroll
              for (int e = 0; e < 16; e += 4)
                st_global_v4(dst + e, o[e], o[e + 1], o[e + 2], o[e + 3]);
            }
          }
        }
      }
      if (tma_out) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("bar.sync 1, 128;" ::: "memory");  // the four epilogue warps
        if (threadIdx.x == 128) {
          const int col0 = blockIdx.x * kTcBN;  // relative to the output map's origin
          for (int b = 0; b < kTcBN / 32; b++)
            if (p.nb0 * 16 + col0 + b * 32 < p.n_end)
              tc::tma_store_2d(&tmC, smem + (size_t)b * (kTcBM * 128), col0 + b * 32, m0);
          tc::bulk_commit();
          tc::bulk_wait_read();
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (s_fail && threadIdx.x == 0 && p.err) atomicExch(p.err, 2);
  if (warp == 2) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTcTmemCols);
  }
}

// .fgm int8 tiles -> row-major [N][K]: output word (n, k/4) reads tile word
// (k%64/4, n%16) of tile (n/16, k/64).
__global__ void q8c_tiles_to_rows(const uint32_t *__restrict__ src, uint32_t *__restrict__ dst,
                                  int N, int K) {
  const int KQ = K / 4, KB = K / 64;
  const size_t words = (size_t)N * KQ;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < words;
       i += (size_t)gridDim.x * blockDim.x) {
    const int n = (int)(i / KQ), kq = (int)(i % KQ);
    dst[i] = src[((size_t)(n >> 4) * KB + (kq >> 4)) * 256 + (kq & 15) * 16 + (n & 15)];
  }
}

// Tile-packed activations [ceil(M/16)][K/64][16][64] -> row-major [M][K].
__global__ void packed_a_to_rows(const uint32_t *__restrict__ src, uint32_t *__restrict__ dst,
                                 int M, int K) {
  const int KQ = K / 4, KB = K / 64;
  const size_t words = (size_t)M * KQ;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < words;
       i += (size_t)gridDim.x * blockDim.x) {
    const int m = (int)(i / KQ), kq = (int)(i % KQ);
    dst[i] = src[((size_t)(m >> 4) * KB + (kq >> 4)) * 256 + (m & 15) * 16 + (kq & 15)];
  }
}

// cuTensorMapEncodeTiled, resolved through the runtime (no libcuda link).
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void *f = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  }
  return fn;
}

unsigned grid_for(size_t words) {
  const size_t b = (words + 255) / 256;
  return (unsigned)(b < 8192 ? (b ? b : 1) : 8192);
}

}  // namespace

// Row-major [rows][ld] byte matrix (K = ld valid bytes per row) as a 2-D TMA
// view with boxes of `box_rows` rows x 128 bytes, 128-byte swizzle.
bool encode_rows_map(CUtensorMap *map, const void *base, int rows, int K, int ld, int box_rows) {
  auto enc = get_encode();
  if (!enc) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld};
  const cuuint32_t box[2] = {(cuuint32_t)kTcBK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t launch_q8c_rows(const int8_t *tiles, int8_t *rows, int N, int K, cudaStream_t st) {
  const size_t words = (size_t)N * K / 4;
  q8c_tiles_to_rows<<<grid_for(words), 256, 0, st>>>(reinterpret_cast<const uint32_t *>(tiles),
                                                     reinterpret_cast<uint32_t *>(rows), N, K);
  return cudaGetLastError();
}

cudaError_t launch_packed_to_rows(const int8_t *packed, int8_t *rows, int M, int K,
                                  cudaStream_t st) {
  const size_t words = (size_t)M * K / 4;
  packed_a_to_rows<<<grid_for(words), 256, 0, st>>>(reinterpret_cast<const uint32_t *>(packed),
                                                    reinterpret_cast<uint32_t *>(rows), M, K);
  return cudaGetLastError();
}

size_t q8c_tc_smem_bytes(int stages) {
  size_t ring = (size_t)stages * kTcStage;
  const size_t out = (size_t)(kTcBN / 32) * kTcBM * 128;  // staged f32 tile
  if (ring < out) ring = out;
  return ring + (size_t)(2 * stages + 1) * 8 + 16 + 1024;
}

// f32 output region [rows][cols] at base (row pitch ld bytes) as a 2-D TMA
// view for stores: boxes of 256 rows x 32 floats, 128-byte swizzle.
static bool encode_out_map(CUtensorMap *map, void *base, int rows, int cols, size_t ld) {
  auto enc = get_encode();
  if (!enc) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld};
  const cuuint32_t box[2] = {32, (cuuint32_t)kTcBM};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t launch_q8c_tc(const TcParams &p_in, int lda, const CUtensorMap &tmB, bool pdl,
                          cudaStream_t st) {
  TcParams p = p_in;
  CUtensorMap tmA, tmC;
  if (!encode_rows_map(&tmA, p.A, p.M, p.K, lda, kTcBM)) return cudaErrorInvalidValue;
  // TMA stores need a 16-byte aligned origin and row pitch
  float *origin = p.C ? p.C + (p.nb0 * 16 - p.c_col0) : nullptr;
  p.tma_store = !p.acc && p.C && ((uintptr_t)origin & 15) == 0 && (p.ldc % 4) == 0 &&
                encode_out_map(&tmC, origin, p.M, p.n_end - p.nb0 * 16, (size_t)p.ldc * 4);
  if (!p.tma_store) memset(&tmC, 0, sizeof(tmC));
  const size_t smem = q8c_tc_smem_bytes(p.stages);
  cudaError_t e = cudaFuncSetAttribute(q8c_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  const int ncols = p.n_end - p.nb0 * 16;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((ncols + kTcBN - 1) / kTcBN, (p.M + kTcBM - 1) / kTcBM);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, q8c_tc_kernel, tmA, tmB, tmC, p);
}

}  // namespace fgm
