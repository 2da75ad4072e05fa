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
// One CTA owns a BM x NB output tile -- 128 x 256 (N=256 MMAs: the fewest
// operand bytes per MAC), 256 x 128 (two M=128 halves sharing each B tile)
// or 128 x 128 (when K must be split) -- and walks its K range in 128-byte
// stages through a 4-deep ring: warp
// 0 (one lane) issues the TMA loads, warp 1 (one lane) issues four K=32 MMAs
// per half per stage and commits each stage back to the producer, warp 2 owns
// the tensor-memory allocation; then all eight warps drain the accumulators
// (tcgen05.ld, each warp its TMEM lane quadrant and half of the columns) and
// apply the f32 epilogue, staged in shared memory for TMA stores.
//
// When the output has too few tiles to occupy the SMs (the 8192 x 2048 down
// projection has 16), a cluster of up to 8 CTAs splits each tile's K range.
// The int32 partial tiles meet in the CTAs' idle operand rings: after a
// cluster barrier every CTA pushes each partial row into the shared memory of
// the CTA that owns it (rows z*BM/splits.. belong to CTA z), which sums them
// after a second barrier.  Integer addition is exact in any order, so the
// result is bit-identical to the unsplit sum.  Every mbarrier wait is bounded
// in time; a kernel that gives up sets the device error flag, still reaches
// every cluster barrier and releases its tensor memory.

#include <cuda.h>

#include <atomic>
#include <cstring>

#include "fgm_common.cuh"
#include "fgm_internal.h"
#include "tc_ptx.cuh"

namespace fgm {

namespace {

constexpr int kTcBMax = 256;  // at most two M=128 halves per tile
constexpr int kTcBN = 128;     // tile width of the split-capable tiles
constexpr int kTcBNMax = 256;  // widest tile (one M=128 half, N=256 MMAs)
constexpr int kTcBK = 128;     // bytes of K per stage
constexpr int kTcThreads = 256;
static_assert(kTcThreads == kTcBMax && kTcThreads == kTcBNMax,
              "one thread per tile row / column loads the scales");

// Tile geometry for H M-halves of 128 rows (H = 1 or 2) and NB columns (128,
// or 256 with H = 1: N=256 MMAs read a quarter fewer operand bytes per MAC
// from shared memory and halve the MMA count).
template <int H, int NB = kTcBN>
struct TcTile {
  static_assert(NB == 128 || (NB == 256 && H == 1), "tile shapes: 128/256 x 128, 128 x 256");
  static constexpr int BM = 128 * H;
  static constexpr int A = BM * kTcBK;          // activation bytes per stage
  static constexpr int Stage = A + NB * kTcBK;  // bytes per ring stage
  static constexpr int TmemCols = H * NB;       // int32 accumulator columns
  static constexpr size_t Out = (size_t)(NB / 32) * BM * 128;  // staged output tile
};

__device__ __forceinline__ void st_global_v4(float *p, float a, float b, float c, float d) {
  asm volatile("st.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

// Split-K buffers in the idle operand ring, int32 rows of 512 bytes (32
// sixteen-byte chunks, chunk c of row r stored at chunk c ^ (r & 7):
// conflict-free for the per-row writes and the per-chunk reads):
//   send  [BM rows]: this CTA's partial tile; rows [j*R, (j+1)*R) go to CTA j
//   recv  [splits-1 slots][R rows] at BM*512: the other CTAs' partials of
//         this CTA's own rows [z*R, (z+1)*R), slot (j < z ? j : j - 1).
__device__ __forceinline__ uint32_t row_off(int r, int chunk) {
  return (uint32_t)(r * 512 + ((chunk ^ (r & 7)) << 4));
}

template <int H, int NB>
__global__ void __launch_bounds__(kTcThreads, 1)
    q8c_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                  const __grid_constant__ CUtensorMap tmC, const TcParams p) {
  using T = TcTile<H, NB>;
  constexpr int BM = T::BM;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // stage buffers must sit on 1 KB boundaries for the swizzle pattern
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int S = p.stages;
  const size_t ring = (size_t)S * T::Stage > T::Out ? (size_t)S * T::Stage : T::Out;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + ring);
  uint64_t *empty = full + S;
  uint64_t *accum = empty + S;
  uint64_t *recv_bar = accum + 1;  // split K: the peers' partials have landed
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(recv_bar + 1);
  __shared__ int s_fail, s_any_fail;
  __shared__ float s_as[kTcBMax];  // a_scale of the tile's rows
  __shared__ float s_bs[NB];  // b_scale of the tile's columns

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KS = (p.K + kTcBK - 1) / kTcBK;
  // tile coordinates: with m_fast the CTAs that run together share their
  // weight tile (B streams from HBM once; the activations stay in L2)
  const int tile_n = p.m_fast ? blockIdx.y : blockIdx.x;
  const int m0 = (p.m_fast ? blockIdx.x : blockIdx.y) * BM;
  const int n0 = p.nb0 * 16 + tile_n * NB;
  // K slice of this CTA: the cluster's CTAs split the tile's K range evenly
  const int splits = p.splits, z = splits > 1 ? (int)tc::cluster_ctarank() : 0;
  const int ks0 = (int)((long)KS * z / splits), ks1 = (int)((long)KS * (z + 1) / splits);
  const int nks = ks1 - ks0;

  if (threadIdx.x == 0) {
    s_fail = 0;
    for (int s = 0; s < S; s++) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    tc::mbar_init(accum, 1);
    tc::mbar_init(recv_bar, 1);
    tc::fence_mbar_init();
    tc::prefetch_tmap(&tmA);
    tc::prefetch_tmap(&tmB);
  }
  if (threadIdx.x < NB) {  // weight scales do not depend on earlier kernels
    const int n = n0 + threadIdx.x;
    s_bs[threadIdx.x] = (p.b_scale && n < p.n_end) ? p.b_scale[n] : 0.0f;
  }
  if (warp == 2) {
    tc::tmem_alloc(tmem_slot, T::TmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == 0 && lane == 0) {  // ---------------------------------- producer
    auto load_b = [&](uint8_t *sa, int i, int s) {
      tc::tma_load_2d(sa + T::A, &tmB, &full[s], (ks0 + i) * kTcBK, n0);
      if (NB == 256)  // the weight map's boxes are 128 rows: the second half
        tc::tma_load_2d(sa + T::A + 128 * kTcBK, &tmB, &full[s], (ks0 + i) * kTcBK, n0 + 128);
    };
    // The weights do not come from earlier kernels: the first ring fill's
    // weight boxes go out before griddepcontrol.wait (each stage's barrier
    // already expects its activation box too), overlapping the predecessor.
    const int pre = nks < S ? nks : S;
    for (int i = 0; i < pre; i++) {
      uint8_t *sa = smem + (size_t)i * T::Stage;
      tc::mbar_expect_tx(&full[i], T::Stage);
      load_b(sa, i, i);
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");  // activations from earlier kernels
    for (int i = 0; i < pre; i++)
      tc::tma_load_2d(smem + (size_t)i * T::Stage, &tmA, &full[i], (ks0 + i) * kTcBK, m0);
    for (int i = pre; i < nks; i++) {
      const int s = i % S;
      if (!tc::mbar_wait(&empty[s], ((i / S) & 1) ^ 1)) {
        s_fail = 1;
        break;
      }
      uint8_t *sa = smem + (size_t)s * T::Stage;
      tc::mbar_expect_tx(&full[s], T::Stage);
      tc::tma_load_2d(sa, &tmA, &full[s], (ks0 + i) * kTcBK, m0);
      load_b(sa, i, s);
    }
  } else if (warp == 1 && lane == 0) {  // ---------------------------- MMA
    const uint32_t idesc = tc::idesc_i8(128, NB);
    for (int i = 0; i < nks; i++) {
      const int s = i % S;
      if (!tc::mbar_wait(&full[s], (i / S) & 1)) {
        s_fail = 1;
        break;
      }
      tc::fence_after_sync();
      const uint32_t sa = tc::smem_u32(smem + (size_t)s * T::Stage);
      const uint32_t sb = sa + T::A;
#pragma unroll
      for (int h = 0; h < H; h++)
#pragma unroll
        for (int j = 0; j < kTcBK / 32; j++)  // K=32 slices of the 128-byte stage
          tc::mma_i8(tmem + h * NB, tc::sdesc_sw128(sa + h * 128 * kTcBK + j * 32),
                     tc::sdesc_sw128(sb + j * 32), idesc, (i | j) != 0);
      tc::mma_commit(&empty[s]);  // stage s is free once these MMAs complete
    }
    tc::mma_commit(accum);
  }
  __syncwarp();

  // ------------------------------------------------------------ epilogue
  // All eight warps drain the accumulators: warp w reads TMEM lane quadrant
  // w % 4 (rows 32(w%4).. of each M half) and the column half w / 4 (NB/2
  // columns, in passes of 64).
  const bool ok = __all_sync(0xffffffffu, tc::mbar_wait(accum, 0));  // warp-uniform
  if (!ok) s_fail = 1;
  tc::fence_after_sync();
  if constexpr (NB == 128) {
    // split K: this CTA's int32 partial goes into its send buffer before the
    // cluster barrier -- its ring is idle once its own MMAs are done, and the
    // peers write only into its receive slots, only after the barrier -- so
    // the drain overlaps the wait for the slowest CTA of the cluster
    if (splits > 1 && ok) {
      const int q = warp & 3, ch = warp >> 2;
#pragma unroll 1
      for (int h = 0; h < H; h++) {
        const int ml = h * 128 + q * 32 + lane;
        uint32_t v[64];
        const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + h * NB + ch * (NB / 2);
        tc::tmem_ld_x32(ta, v);
        tc::tmem_ld_x32(ta + 32, v + 32);
        tc::tmem_wait_ld();
#pragma unroll
        for (int c4 = 0; c4 < 16; c4++)
          *reinterpret_cast<uint4 *>(smem + row_off(ml, ch * 16 + c4)) =
              make_uint4(v[4 * c4], v[4 * c4 + 1], v[4 * c4 + 2], v[4 * c4 + 3]);
      }
    }
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");  // a_scale comes from earlier kernels
  if (threadIdx.x < BM) {
    const int m = m0 + threadIdx.x;
    s_as[threadIdx.x] = (p.a_scale && m < p.M) ? p.a_scale[m] : 0.0f;
  }
  __syncthreads();
  // split K: every CTA of the cluster is past its main loop (its ring is free
  // to receive partials, its failure flag final) before anyone pushes
  if (splits > 1) {
    // expect every peer's copy before anyone can send one
    if (threadIdx.x == 0)
      tc::mbar_expect_tx(recv_bar, (uint32_t)((splits - 1) * (BM / splits) * 512));
    tc::cluster_sync();
    if (threadIdx.x == 0) {  // did any CTA of the cluster fail?
      int any = 0;
      for (int src = 0; src < splits; src++) {
        int f;
        asm volatile("ld.shared::cluster.u32 %0, [%1];"
                     : "=r"(f)
                     : "r"(tc::mapa(tc::smem_u32(&s_fail), (uint32_t)src))
                     : "memory");
        any |= f;
      }
      s_any_fail = any;
    }
  }
  const int q = warp & 3, ch = warp >> 2;
  const bool tma_out = p.tma_store != 0;  // launcher: no raw output, no split, aligned
  if (ok && !s_fail && splits == 1) {  // (a split CTA drained its partial above)
#pragma unroll 1
    for (int h = 0; h < H; h++) {
      const int ml = h * 128 + q * 32 + lane;
      const int m = m0 + ml;
      const bool row_ok = m < p.M;
      const float as = s_as[ml];
#pragma unroll 1
      for (int cb = 0; cb < NB / 128; cb++) {  // 64 of this warp's NB/2 columns per pass
      uint32_t v[64];
      const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + h * NB + ch * (NB / 2) + cb * 64;
      tc::tmem_ld_x32(ta, v);
      tc::tmem_ld_x32(ta + 32, v + 32);
      tc::tmem_wait_ld();
#pragma unroll
      for (int cc = 0; cc < 4; cc++) {
        const int c = ch * (NB / 32) + cb * 4 + cc;  // 16-column chunk of the tile
        const int n = n0 + c * 16;
        if (p.acc) {
          if (row_ok && n < p.n_end)
            for (int e = 0; e < 16; e++) p.acc[(size_t)m * p.N + n + e] = (int32_t)v[cc * 16 + e];
          continue;
        }
        if (n >= p.n_end) continue;
        float o[16];
#pragma unroll
        for (int e = 0; e < 16; e++)
          o[e] = __fmul_rn(__int2float_rn((int32_t)v[cc * 16 + e]), __fmul_rn(s_bs[c * 16 + e], as));
        if (tma_out) {
          uint8_t *rowp = smem + (size_t)(c >> 1) * (BM * 128) + (size_t)ml * 128;
#pragma unroll
          for (int t = 0; t < 4; t++) {
            const int j = (c & 1) * 4 + t;  // 16-byte chunk inside the 128-byte row
            *reinterpret_cast<float4 *>(rowp + ((j ^ (ml & 7)) << 4)) =
                make_float4(o[4 * t], o[4 * t + 1], o[4 * t + 2], o[4 * t + 3]);
          }
        } else if (row_ok) {
          float *dst = p.C + (size_t)m * p.ldc + (n - p.c_col0);
          if (p.out_v4) {
#pragma unroll
            for (int e = 0; e < 16; e += 4) st_global_v4(dst + e, o[e], o[e + 1], o[e + 2], o[e + 3]);
          } else {
#pragma unroll
            for (int e = 0; e < 16; e++) dst[e] = o[e];
          }
        }
      }
      if constexpr (NB == 256) {
        // 256-wide tiles drain in two passes; the four 32-column blocks a pass
        // completed go out while the next pass drains.  The branch is
        // block-uniform here (a warp whose accumulator wait failed raised
        // s_fail before the barrier above), so the block barrier is safe.
        if (tma_out) {
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncthreads();
          if (threadIdx.x == 0) {
            const int col0 = tile_n * NB;  // relative to the output map's origin
            for (int half = 0; half < 2; half++)
              for (int b2 = 0; b2 < 2; b2++) {
                const int b = half * 4 + cb * 2 + b2;  // 32-column block of the tile
                if (p.nb0 * 16 + col0 + b * 32 < p.n_end)
                  tc::tma_store_2d(&tmC, smem + (size_t)b * (BM * 128), col0 + b * 32, m0);
              }
            tc::bulk_commit();
          }
        }
      }
      }
    }
  }
  if (tma_out) {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (threadIdx.x == 0 && ok && !s_fail) {
      if constexpr (NB == 128) {  // (256-wide tiles stored theirs pass by pass)
        const int col0 = tile_n * NB;  // relative to the output map's origin
        for (int b = 0; b < NB / 32; b++)
          if (p.nb0 * 16 + col0 + b * 32 < p.n_end)
            tc::tma_store_2d(&tmC, smem + (size_t)b * (BM * 128), col0 + b * 32, m0);
        tc::bulk_commit();
      }
      tc::bulk_wait_read();
    }
  }
  if constexpr (NB == 128) {
  if (splits > 1) {
    // One bulk copy per peer moves the rows it owns from this CTA's send
    // buffer into its receive slot (completing on its mbarrier); then CTA z
    // sums rows [z*R, (z+1)*R) over its own partial and the received ones
    // (int32, exact in any order), scales them and stores them.  Copies go
    // out even from a failed CTA so no receiver is left waiting; if any CTA
    // failed, the cluster skips the stores and the flag is raised.  The last
    // barrier keeps every send buffer alive until its copies have landed.
    const int R = BM / splits;
    const uint32_t send = tc::smem_u32(smem), recv = send + (uint32_t)BM * 512;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // partials -> copy engine
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int j = 0; j < splits; j++) {
        if (j == z) continue;
        const int slot = z < j ? z : z - 1;
        tc::bulk_s2cluster(tc::mapa(recv + (uint32_t)(slot * R * 512), (uint32_t)j),
                           send + (uint32_t)(j * R * 512), (uint32_t)(R * 512),
                           tc::mapa(tc::smem_u32(recv_bar), (uint32_t)j));
      }
    }
    const bool got = __all_sync(0xffffffffu, tc::mbar_wait(recv_bar, 0));
    if (!got) s_fail = 1;
    __syncthreads();
    const int fail_any = s_any_fail || s_fail;
    for (int sl = threadIdx.x; sl < R * 32; sl += kTcThreads) {
      const int rl = sl / 32, chunk = sl % 32;
      const int m = m0 + z * R + rl, n = n0 + chunk * 4;
      uint4 acc = *reinterpret_cast<const uint4 *>(smem + row_off(z * R + rl, chunk));
      for (int slot = 0; slot < splits - 1; slot++) {
        const uint4 u = *reinterpret_cast<const uint4 *>(smem + BM * 512 + slot * R * 512 +
                                                         row_off(rl, chunk));
        acc.x += u.x;
        acc.y += u.y;
        acc.z += u.z;
        acc.w += u.w;
      }
      if (fail_any || m >= p.M || n >= p.n_end) continue;
      const uint32_t a4[4] = {acc.x, acc.y, acc.z, acc.w};
      if (p.acc) {
        for (int e = 0; e < 4; e++) p.acc[(size_t)m * p.N + n + e] = (int32_t)a4[e];
        continue;
      }
      const float as = s_as[z * R + rl];
      float o[4];
#pragma unroll
      for (int e = 0; e < 4; e++)
        o[e] = __fmul_rn(__int2float_rn((int32_t)a4[e]), __fmul_rn(s_bs[chunk * 4 + e], as));
      float *dst = p.C + (size_t)m * p.ldc + (n - p.c_col0);
      if (p.out_v4)
        st_global_v4(dst, o[0], o[1], o[2], o[3]);
      else
        for (int e = 0; e < 4; e++) dst[e] = o[e];
    }
    tc::cluster_sync();
  }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (s_fail && threadIdx.x == 0 && p.err) atomicExch(p.err, 2);
  if (warp == 2) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, T::TmemCols);
  }
}

// ------------------------------------------------- persistent 128 x 256 tiles
// For outputs with more 128 x 256 tiles than SMs: one CTA per SM walks the
// tiles (M tiles fastest, so the CTAs running together share weight tiles)
// with two int32 accumulators in tensor memory (2 x 256 of the 512 columns),
// so one tile's epilogue overlaps the next tile's MMAs.  Warp 0 (one lane)
// streams the A / B stages of every tile through the ring; warp 1 (one lane)
// issues the MMAs of tile i into accumulator i % 2 once the epilogue has
// drained that accumulator (tile i - 2) and commits it; warps 4-7 drain an
// accumulator (warp w: TMEM lanes 32(w%4)..), scale it and write the tile
// through two 16 KB staging buffers of 32 columns with TMA stores.  Each
// staging buffer is rewritten only after the store that last read it is
// done reading.  Every wait is bounded; a warp that gives up raises the
// flag, and the producer lets the loads it issued land before the CTA ends.
constexpr int kTpStage = 128 * kTcBK + 256 * kTcBK;  // A 128 rows + B 256 rows
constexpr int kTpOut = 128 * 128;                    // 32 f32 columns x 128 rows

__device__ __forceinline__ void epi_sync() {  // the four epilogue warps
  asm volatile("bar.sync 2, 128;" ::: "memory");
}

// True on every epilogue thread when any of them passes true.
__device__ __forceinline__ bool epi_any(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 2, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v)
      : "memory");
  return r != 0;
}

__global__ void __launch_bounds__(kTcThreads, 1)
    q8c_tc_persistent(const __grid_constant__ CUtensorMap tmA,
                      const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmC, const TcParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int S = p.stages;
  uint8_t *stage_out = smem + (size_t)S * kTpStage;  // 2 x kTpOut
  uint64_t *full = reinterpret_cast<uint64_t *>(stage_out + 2 * kTpOut);
  uint64_t *empty = full + S;
  uint64_t *tfull = empty + S;   // [2] accumulator b holds a finished tile
  uint64_t *tempty = tfull + 2;  // [2] accumulator b is drained (4 epilogue warps arrive)
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tempty + 2);
  __shared__ int s_fail;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KS = (p.K + kTcBK - 1) / kTcBK;
  const int ncols = p.n_end - p.nb0 * 16;
  const int mt = (p.M + 127) / 128, nt = (ncols + 255) / 256;
  const int tiles = mt * nt;

  if (threadIdx.x == 0) {
    s_fail = 0;
    for (int s = 0; s < S; s++) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      tc::mbar_init(&tfull[b], 1);
      tc::mbar_init(&tempty[b], 4);
    }
    tc::fence_mbar_init();
    tc::prefetch_tmap(&tmA);
    tc::prefetch_tmap(&tmB);
    tc::prefetch_tmap(&tmC);
  }
  if (warp == 2) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == 0) {  // ------------------------------------------------ producer
    if (lane == 0) {
      asm volatile("griddepcontrol.wait;" ::: "memory");  // activations from earlier kernels
      uint32_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const int m0 = (t % mt) * 128, n0 = p.nb0 * 16 + (t / mt) * 256;
        for (int k = 0; k < KS; k++, it++) {
          const int s = (int)(it % S);
          if (!tc::mbar_wait(&empty[s], ((it / S) & 1) ^ 1)) {
            ok = false;
            break;
          }
          uint8_t *sa = smem + (size_t)s * kTpStage;
          tc::mbar_expect_tx(&full[s], kTpStage);
          tc::tma_load_2d(sa, &tmA, &full[s], k * kTcBK, m0);
          tc::tma_load_2d(sa + 128 * kTcBK, &tmB, &full[s], k * kTcBK, n0);
          tc::tma_load_2d(sa + 256 * kTcBK, &tmB, &full[s], k * kTcBK, n0 + 128);
        }
      }
      if (!ok) {
        s_fail = 1;
        // the last loads issued land before the CTA can end
        for (uint32_t j = it > (uint32_t)S ? it - S : 0; j < it; j++)
          tc::mbar_wait(&full[j % S], (j / S) & 1, 100000000ull);
      }
    }
  } else if (warp == 1) {  // ------------------------------------------ MMA
    if (lane == 0) {
      const uint32_t idesc = tc::idesc_i8(128, 256);
      uint32_t it = 0, i = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, i++) {
        const uint32_t b = i & 1;
        if (!tc::mbar_wait(&tempty[b], ((i >> 1) & 1) ^ 1)) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
        for (int k = 0; k < KS; k++, it++) {
          const int s = (int)(it % S);
          if (!tc::mbar_wait(&full[s], (it / S) & 1)) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const uint32_t sa = tc::smem_u32(smem + (size_t)s * kTpStage);
          const uint32_t sb = sa + 128 * kTcBK;
#pragma unroll
          for (int j = 0; j < kTcBK / 32; j++)
            tc::mma_i8(tmem + b * 256, tc::sdesc_sw128(sa + j * 32), tc::sdesc_sw128(sb + j * 32),
                       idesc, (k | j) != 0);
          tc::mma_commit(&empty[s]);
        }
        if (ok) tc::mma_commit(&tfull[b]);
      }
      if (!ok) s_fail = 1;
    }
  } else if (warp >= 4) {  // ------------------------------------- epilogue
    const int q = warp & 3, ml = q * 32 + lane, et = threadIdx.x - 128;
    asm volatile("griddepcontrol.wait;" ::: "memory");  // a_scale from earlier kernels
    uint32_t i = 0, sb = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, i++) {
      const uint32_t b = i & 1;
      const int m0 = (t % mt) * 128, tn = t / mt, n0 = p.nb0 * 16 + tn * 256;
      ok = __all_sync(0xffffffffu, tc::mbar_wait(&tfull[b], (i >> 1) & 1));
      // the four warps agree before any of them leaves the named barriers
      if (epi_any(!ok)) {
        ok = false;
        break;
      }
      tc::fence_after_sync();
      const int m = m0 + ml;
      const float as = (p.a_scale && m < p.M) ? p.a_scale[m] : 0.0f;
#pragma unroll 1
      for (int c = 0; c < 8; c++) {  // 32-column chunks
        uint32_t v[32];
        tc::tmem_ld_x32(tmem + ((uint32_t)(q * 32) << 16) + b * 256 + c * 32, v);
        tc::tmem_wait_ld();
        if (c == 7) {  // the accumulator is free for tile i + 2
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&tempty[b]);
        }
        const int nc = n0 + c * 32;
        if (nc >= p.n_end) continue;  // past the last column (uniform over the warps)
        float bs[32];
#pragma unroll
        for (int e = 0; e < 32; e++) bs[e] = nc + e < p.n_end ? __ldg(p.b_scale + nc + e) : 0.0f;
        // staging buffer sb % 2 (sb counts the stores issued): free once the
        // store before the latest one has read it
        if (et == 0) tc::bulk_wait_read_1();
        epi_sync();
        uint8_t *rowp = stage_out + (size_t)(sb & 1) * kTpOut + (size_t)ml * 128;
#pragma unroll
        for (int j = 0; j < 8; j++) {
          float o[4];
#pragma unroll
          for (int e = 0; e < 4; e++)
            o[e] = __fmul_rn(__int2float_rn((int32_t)v[j * 4 + e]), __fmul_rn(bs[j * 4 + e], as));
          *reinterpret_cast<float4 *>(rowp + ((j ^ (ml & 7)) << 4)) =
              make_float4(o[0], o[1], o[2], o[3]);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        epi_sync();
        if (et == 0) {
          tc::tma_store_2d(&tmC, stage_out + (size_t)(sb & 1) * kTpOut, tn * 256 + c * 32, m0);
          tc::bulk_commit();
        }
        sb++;
      }
    }
    if (!ok) s_fail = 1;
    if (et == 0) tc::bulk_wait_all();
  }
  tc::fence_before_sync();
  __syncthreads();
  if (s_fail && threadIdx.x == 0 && p.err) atomicExch(p.err, 2);
  if (warp == 2) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, 512);
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

// Tile-packed activations [1][K/64][16][64] (M <= 16) as a 3-D TMA view
// (64 bytes, 16 rows, K/64 tiles) read in one box of `rows` rows x every tile,
// with the 64-byte swizzle: 16-byte chunk c of row r lands at chunk
// c ^ ((r >> 1) & 3) of its 64-byte shared-memory row.
bool encode_packed_a_map(CUtensorMap *map, const void *base, int K, int rows) {
  auto enc = get_encode();
  if (!enc || K % 64 != 0 || K / 64 > 256 || rows < 1 || rows > 16) return false;
  const cuuint64_t dims[3] = {64, 16, (cuuint64_t)(K / 64)};
  const cuuint64_t strides[2] = {64, 1024};
  const cuuint32_t box[3] = {64, (cuuint32_t)rows, (cuuint32_t)(K / 64)};
  const cuuint32_t estr[3] = {1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// int4 group scales f16 [groups][N] as a 2-D TMA view, boxes of 16 columns x
// `rows` group rows (one 32-byte row per group), no swizzle.
bool encode_scale_map(CUtensorMap *map, const void *base, int groups, int N, int rows) {
  auto enc = get_encode();
  if (!enc || N % 16 != 0 || rows < 1 || rows > 8) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)groups};
  const cuuint64_t strides[1] = {(cuuint64_t)N * 2};
  const cuuint32_t box[2] = {16, (cuuint32_t)rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void *>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
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

template <int H, int NB = kTcBN>
size_t tc_smem_bytes(int stages) {
  using T = TcTile<H, NB>;
  size_t ring = (size_t)stages * T::Stage;
  if (ring < T::Out) ring = T::Out;
  return ring + (size_t)(2 * stages + 2) * 8 + 16 + 1024;
}

constexpr size_t kTcStaticReserve = 4096;  // the kernel's static shared memory (about 2 KB)

template <int H, int NB = kTcBN>
int tc_stages(size_t smem_limit) {
  int st = 8;
  while (st > 2 && tc_smem_bytes<H, NB>(st) + kTcStaticReserve > smem_limit) st--;
  return st;
}

// Clusters of `s` CTAs of kernel<H> that can be resident at once (cached).
template <int H>
int tc_max_clusters(int s, size_t smem) {
  static std::atomic<int> cache[9];
  int v = cache[s].load(std::memory_order_relaxed);
  if (v > 0) return v;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1, 1, s);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = (unsigned)s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaFuncSetAttribute(q8c_tc_kernel<H, kTcBN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess ||
      cudaOccupancyMaxActiveClusters(&v, q8c_tc_kernel<H, kTcBN>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    v = 0;  // unknown: no split for this size
  }
  cache[s].store(v > 0 ? v : -1, std::memory_order_relaxed);
  return v;
}

// Tile height and K split for a launch.  Every candidate runs in one wave
// (split launches: all clusters resident at once; unsplit: waves counted);
// the choice minimises the operand bytes one CTA must stream per wave,
// since the main loop is bound by each SM's load throughput.
struct TcChoice {
  int H, splits, stages;
  size_t smem;
  int NB;
};

TcChoice plan_tc(int M, int ncols, int K, int num_sms, size_t smem_limit) {
  const int KS = (K + kTcBK - 1) / kTcBK;
  TcChoice best{2, 1, tc_stages<2>(smem_limit), 0, kTcBN};
  best.smem = tc_smem_bytes<2>(best.stages);
  double best_cost = -1;
  {  // 128 x 256 tiles first: on a tie in operand bytes the N=256 MMAs win
    const int stages = tc_stages<1, 256>(smem_limit);
    const size_t smem = tc_smem_bytes<1, 256>(stages);
    const long tiles = (long)((ncols + 255) / 256) * ((M + 127) / 128);
    const double waves = (double)((tiles + num_sms - 1) / num_sms);
    best_cost = waves * (double)(128 + 256) * K;
    best = TcChoice{1, 1, stages, smem, 256};
  }
  for (int H = 2; H >= 1; H--) {
    const int stages = H == 2 ? tc_stages<2>(smem_limit) : tc_stages<1>(smem_limit);
    const size_t smem = H == 2 ? tc_smem_bytes<2>(stages) : tc_smem_bytes<1>(stages);
    const long tiles = (long)((ncols + kTcBN - 1) / kTcBN) * ((M + 128 * H - 1) / (128 * H));
    for (int s = 1; s <= 8; s *= 2) {
      if (s > 1 && KS < 4 * s) break;
      // split K stages the send tile and the received slots in the ring
      const size_t ring = (size_t)stages * (size_t)(128 * H + kTcBN) * kTcBK;
      if (s > 1 && (size_t)(128 * H) * 512 * (2 * s - 1) / s > ring) continue;
      const long ctas = tiles * s;
      double waves;
      if (s == 1) {
        waves = (double)((ctas + num_sms - 1) / num_sms);
      } else {
        if (ctas > num_sms) break;
        const int mc = H == 2 ? tc_max_clusters<2>(s, smem) : tc_max_clusters<1>(s, smem);
        if (tiles > mc) continue;
        waves = 1.0;
      }
      const double cost = waves * (double)(128 * H + kTcBN) * ((double)K / s);
      if (best_cost < 0 || cost < best_cost * 0.999) {
        best_cost = cost;
        best = TcChoice{H, s, stages, smem, kTcBN};
      }
    }
  }
  return best;
}

// f32 output region [rows][cols] at base (row pitch ld bytes) as a 2-D TMA
// view for stores: boxes of 256 rows x 32 floats, 128-byte swizzle.
static bool encode_out_map(CUtensorMap *map, void *base, int rows, int cols, size_t ld,
                           int box_rows) {
  auto enc = get_encode();
  if (!enc) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld};
  const cuuint32_t box[2] = {32, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t tp_smem_bytes(int stages) {
  return (size_t)stages * kTpStage + 2 * (size_t)kTpOut + (size_t)(2 * stages + 4) * 8 + 16 + 1024;
}

// The persistent kernel when it applies (128 x 256 tiles, no K split, TMA
// stores, more tiles than SMs); false: use the one-tile-per-CTA kernel.
// FGM_CUDA_TC_PERSISTENT=0 turns it off.
static bool launch_tc_persistent(const TcParams &p, const CUtensorMap &tmA, const CUtensorMap &tmB,
                                 const CUtensorMap &tmC, int num_sms, size_t smem_limit, bool pdl,
                                 cudaStream_t st, cudaError_t *err) {
  static const int enabled = [] {
    const char *e = getenv("FGM_CUDA_TC_PERSISTENT");
    return e ? atoi(e) : 1;
  }();
  const int ncols = p.n_end - p.nb0 * 16;
  const long tiles = (long)((p.M + 127) / 128) * ((ncols + 255) / 256);
  if (!enabled || p.splits != 1 || !p.tma_store || p.acc || tiles <= num_sms) return false;
  int stages = 6;
  static const size_t stat = [] {  // the kernel's static shared memory
    cudaFuncAttributes a{};
    if (cudaFuncGetAttributes(&a, q8c_tc_persistent) != cudaSuccess) {
      cudaGetLastError();
      return (size_t)4096;
    }
    return (size_t)a.sharedSizeBytes;
  }();
  // smem_limit is the opt-in size less 1 KB of headroom for static shared
  // memory; the static size is counted exactly here instead
  const size_t optin = smem_limit + 1024;
  while (stages > 2 && tp_smem_bytes(stages) + stat > optin) stages--;
  const size_t smem = tp_smem_bytes(stages);
  if (smem + stat > optin) return false;
  TcParams q = p;
  q.stages = stages;
  *err = cudaFuncSetAttribute(q8c_tc_persistent, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)smem);
  if (*err != cudaSuccess) return true;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(tiles < num_sms ? tiles : num_sms));
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  *err = cudaLaunchKernelEx(&cfg, q8c_tc_persistent, tmA, tmB, tmC, q);
  return true;
}

template <int H, int NB>
cudaError_t launch_tc_h(const TcParams &p, const CUtensorMap &tmA, const CUtensorMap &tmB,
                        const CUtensorMap &tmC, size_t smem, bool pdl, cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(q8c_tc_kernel<H, NB>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int ncols = p.n_end - p.nb0 * 16;
  const unsigned nt = (unsigned)((ncols + NB - 1) / NB), mt = (unsigned)((p.M + 128 * H - 1) / (128 * H));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = p.m_fast ? dim3(mt, nt, p.splits) : dim3(nt, mt, p.splits);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (p.splits > 1) {  // the CTAs splitting one tile's K form a cluster
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = (unsigned)p.splits;
    na++;
  }
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    na++;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, q8c_tc_kernel<H, NB>, tmA, tmB, tmC, p);
}

cudaError_t launch_q8c_tc(const TcParams &p_in, int lda, const CUtensorMap &tmB, bool pdl,
                          int num_sms, size_t smem_limit, cudaStream_t st) {
  TcParams p = p_in;
  const TcChoice c = plan_tc(p.M, p.n_end - p.nb0 * 16, p.K, num_sms, smem_limit);
  if (c.smem + kTcStaticReserve > smem_limit) return cudaErrorInvalidConfiguration;
  p.stages = c.stages;
  p.splits = c.splits;
  // M tiles fastest when there are several and no K split: a wave's CTAs then
  // share weight tiles instead of each streaming its own
  p.m_fast = c.splits == 1 && p.M > 128 * c.H;
  const int BM = 128 * c.H;
  CUtensorMap tmA, tmC;
  if (!encode_rows_map(&tmA, p.A, p.M, p.K, lda, BM)) return cudaErrorInvalidValue;
  // TMA and vector stores need 16-byte aligned rows
  float *origin = p.C ? p.C + (p.nb0 * 16 - p.c_col0) : nullptr;
  p.out_v4 = p.C && ((uintptr_t)origin & 15) == 0 && (p.ldc % 4) == 0;
  p.tma_store = !p.acc && p.out_v4 && p.splits == 1 &&
                encode_out_map(&tmC, origin, p.M, p.n_end - p.nb0 * 16, (size_t)p.ldc * 4, BM);
  if (!p.tma_store) memset(&tmC, 0, sizeof(tmC));
  if (c.NB == 256) {
    cudaError_t e = cudaSuccess;
    if (launch_tc_persistent(p, tmA, tmB, tmC, num_sms, smem_limit, pdl, st, &e)) return e;
    return launch_tc_h<1, 256>(p, tmA, tmB, tmC, c.smem, pdl, st);
  }
  return c.H == 2 ? launch_tc_h<2, kTcBN>(p, tmA, tmB, tmC, c.smem, pdl, st)
                  : launch_tc_h<1, kTcBN>(p, tmA, tmB, tmC, c.smem, pdl, st);
}

}  // namespace fgm
