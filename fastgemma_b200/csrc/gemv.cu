// Decode-shaped quantised GEMM: C[M, N] for M <= 16 rows per CTA row block,
// reading the .fgm weight tiles exactly as the converter wrote them.
//
// Reference: fgm_gemm_q4g / fgm_gemm_q8c (amx_gemm.c:333-475, small-M path
// INNER_Q4_1x4 :300-331) and their VNNI twins (vnni_gemm.c:224-322).
//
// Why the tile layout needs no repack for the tensor cores
// --------------------------------------------------------
// mma.sync.m16n8k32 (s8) takes its A operand as four 32-bit registers per
// thread; thread (g, t) of a warp (g = lane/4, t = lane%4) holds rows g and
// g+8, k-quads t and 4+t.  With the weights as A (16 output channels x 32 k)
// and the activations as B (32 k x 8 batch rows):
//  * int8 tile row r (64 bytes) holds, at byte 4n, the four k = 4r..4r+3 of
//    channel n (convert/quant.py:96-107), so the word (r, n) is one register;
//  * int4 tile row r (32 bytes) holds, at byte 4q, channel q in the low
//    nibbles and channel q+8 in the high nibbles of the same four k
//    (quant.py:76-82), so ONE 32-bit word yields a row-g and a row-g+8
//    register after a mask: (w << 4) & 0xF0F0F0F0 and w & 0xF0F0F0F0.
// The int4 registers carry 16 * value (nibble in the high half of its byte,
// two's complement), so the int32 sums are 16x the true ones; the factor is
// taken out of the scale (s * 2^-4, exact) or shifted out exactly.
//
// Memory pipeline
// ---------------
// The kernel is persistent.  The work unit is one n-block (16 output columns)
// over all of K; a "team" of P warps shares a unit, warp p taking the p-th
// group-aligned slice of K (P = 1 for wide N, more when N has too few
// n-blocks to occupy every warp).  Each warp streams its slices through a
// private ring of shared-memory stages, one cp.async.bulk per stage (a
// unit's tiles are contiguous in the [N/16][K/64] order, so a stage of 8
// int4 tiles is one 4 KB copy), refilled as soon as a stage is consumed,
// across unit boundaries.  The f16 scale rows do not go through the copy
// engine: each lane loads one 32-bit word of the rows a stage needs, two
// stages ahead, and the values reach their users by warp shuffles.  Weight
// prefetch does not depend on earlier kernels: under programmatic dependent
// launch the ring fills before griddepcontrol.wait, which guards only
// activation reads and output writes.  The activations of the CTA's row
// block are staged once in shared memory in the order the B fragments want
// (k-quads t, 4+t, 8+t, 12+t adjacent): one 128-bit load per tile and 8 rows.
//
// Reduction order and bit-exactness
// ---------------------------------
// Tiles are summed per scale group in int32 (exact).  With P = 1 the warp
// folds each completed group into its f32 outputs right away:
// c = fmaf((float)acc_g, s_g, c), ascending g, then c * a_scale -- the drain
// of amx_gemm.c:103-113 and the final scaling of :365-371.  With P > 1 the
// parts publish their int32 group sums in shared memory and the team folds
// all groups of a unit in ascending order once every part is done.  int8:
// acc * (b_scale * a_scale) (amx_gemm.c:399); parts add int32 partials.
// Every f32 operation is an explicit _rn intrinsic.

#include "fgm_common.cuh"
#include "fgm_internal.h"
#include "stream_ptx.cuh"
#include "tc_ptx.cuh"

namespace fgm {

namespace {

using namespace stream;

constexpr int kMaxWarps = 16;
// Words per published row of group values in the split-K exchange area: 16
// columns plus 4 words of padding, so the rows 2*tig (+1) that one store
// instruction's lanes write fall in distinct banks.  For 16-row blocks the
// planner drops the padding (kPubRowDense) when it would cost the launch its
// activation staging or split-K parts; 8-row blocks always pad (compile-time
// stride, immediate offsets).
constexpr int kPubRow = 20;
constexpr int kPubRowDense = 16;

template <bool Q4>
struct Geo {
  static constexpr int TB = Q4 ? kQ4Tile : kQ8Tile;  // bytes per weight tile
  static constexpr int T = Q4 ? 8 : 4;               // tiles per ring stage
};

__device__ __forceinline__ void team_sync(int team, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(team + 1), "r"(nthreads) : "memory");
}

// Fire-and-forget L2 prefetch of [src, src + bytes): no completion to wait
// for, so a late or dropped prefetch only costs a later miss.
__device__ __forceinline__ void prefetch_l2_bulk(const void *src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// This CTA's slice of the next launch's weight regions, 32 KB per prefetch,
// spread over the lanes of one warp.
__device__ __forceinline__ void warm_next(const GemvParams &p, int lane) {
  constexpr size_t kPiece = 32768;
#pragma unroll
  for (int r = 0; r < 2; r++) {
    const size_t total = p.warm_bytes[r] & ~(size_t)15;
    if (total == 0) continue;
    const size_t per = ((total + gridDim.x - 1) / gridDim.x + 15) & ~(size_t)15;
    const size_t lo = (size_t)blockIdx.x * per;
    const size_t hi = lo + per < total ? lo + per : total;
    for (size_t o = lo + (size_t)lane * kPiece; o < hi; o += 32 * kPiece)
      prefetch_l2_bulk(p.warm[r] + o, (uint32_t)(hi - o < kPiece ? hi - o : kPiece));
  }
}

// ------------------------------------------------------ fused all-gather
// Signal words: see GatherParams (counts grow by a known amount per call).
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *a) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
  return v;
}

// Wait until *a >= want, at most 2 s (then false).
__device__ __forceinline__ bool spin_until_geq(const unsigned long long *a, unsigned long long want) {
  if (ld_acquire_sys(a) >= want) return true;
  const uint64_t t0 = tc::globaltimer_ns();
  while (ld_acquire_sys(a) < want) {
    if (tc::globaltimer_ns() - t0 > 2000000000ull) return false;
    __nanosleep(64);
  }
  return true;
}

__device__ __forceinline__ void st_v4_global(float *p, float4 v) {
  asm volatile("st.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}

// One 8-row block of n-block nb, already stored at Cout (this rank's buffer
// of the call's slot), copied to every peer's buffer: lane = (row, 16-byte
// chunk), 64 contiguous bytes per row.
__device__ __forceinline__ void push_rows(const GemvParams &p, float *Cout, int nb, int m0,
                                          int lane) {
  const int m = m0 + (lane >> 2);
  if (m >= p.M) return;
  const size_t off = (size_t)m * p.ldc + (size_t)(nb * 16 - p.c_col0) + (lane & 3) * 4;
  const float4 v = *reinterpret_cast<const float4 *>(Cout + off);
  const size_t shift = (size_t)(Cout - p.g.out[p.g.rank]);
  for (int q = 0; q < p.g.world; q++)
    if (q != p.g.rank) st_v4_global(p.g.out[q] + shift + off, v);
}

// Before a warp's first push of a call: every rank has announced that its
// buffer of this slot is free (bounded; false on time-out).
__device__ __forceinline__ bool peers_free(const GemvParams &p, int slot, unsigned long long uses,
                                           int lane) {
  bool ok = true;
  if (lane == 0)
    ok = spin_until_geq(p.g.sig[p.g.rank] + 2 + slot, (unsigned long long)p.g.world * uses);
  return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
}

// Per-lane constants shared by the stage routines.
struct Lane {
  int g8, tig, lane;
  int pr;          // words per published row (GemvPlan::pub_row)
  uint32_t w_off;  // weight word (row tig, column g8) inside a tile
  uint32_t a_off;  // activation row g8, k-quads t..12+t, inside a tile's 8 rows
};

// One ring stage of NT tiles, NT a compile-time count (no per-tile guards, so
// all of the stage's loads are issued before its MMAs).  MODE 0: fold each
// completed scale group into cf (int4, P = 1).  MODE 1: publish each
// completed group's int32 sum to pub[g][row][col] (int32 output).  MODE 2:
// accumulate into gacc (int8).  MODE 3: publish each completed group's sum
// as the exact f32 the fold will use, with the group's f32 scales (int4 split
// K parts 1..P-1), so the team's serial fold is a load pair and an FMA per
// group.  Stages start on a group boundary (GK divides NT).
template <bool Q4, int MT, int GK, int NT, int MODE>
__device__ __forceinline__ void stage_full(uint32_t st, uint32_t ab, const Lane &L, int g0,
                                           uint32_t sc0, uint32_t sc1, float (&cf)[MT][4],
                                           int32_t (&gacc)[MT][4], int32_t *pub,
                                           uint32_t *pub_sc) {
  constexpr int TB = Geo<Q4>::TB;
  // tiles whose operands are loaded together before their MMAs: the whole
  // stage for 8-row blocks, half of it for 16 (register budget)
  constexpr int CH = (MT == 1 || NT < 8) ? NT : NT / 2;
#pragma unroll
  for (int t0 = 0; t0 < NT; t0 += CH) {
  uint32_t w[CH][Q4 ? 4 : 8];
  uint32_t b[CH][MT][4];
#pragma unroll
  for (int tc = 0; tc < CH; tc++) {
    const int t = t0 + tc;
#pragma unroll
    for (int q = 0; q < 4; q++) {  // tile rows q*4 + tig
      if (Q4) {
        w[tc][q] = lds32(st + t * TB + L.w_off + q * 128);
      } else {
        w[tc][2 * q] = lds32(st + t * TB + L.w_off + q * 256);
        w[tc][2 * q + 1] = lds32(st + t * TB + L.w_off + q * 256 + 32);
      }
    }
#pragma unroll
    for (int mt = 0; mt < MT; mt++) {
      const uint4 v = lds128(ab + (t * MT + mt) * 512 + L.a_off);
      b[tc][mt][0] = v.x;
      b[tc][mt][1] = v.y;
      b[tc][mt][2] = v.z;
      b[tc][mt][3] = v.w;
    }
  }
#pragma unroll
  for (int tc = 0; tc < CH; tc++) {
    const int t = t0 + tc;
    int32_t ta[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; mt++) {
      if (Q4) {
        mma_s8_m16n8k32_c(ta[mt], nib_lo_x16(w[tc][0]), nib_hi_x16(w[tc][0]),
                          nib_lo_x16(w[tc][1]), nib_hi_x16(w[tc][1]), b[tc][mt][0], b[tc][mt][1],
                          0, 0, 0, 0);
        mma_s8_m16n8k32_c(ta[mt], nib_lo_x16(w[tc][2]), nib_hi_x16(w[tc][2]),
                          nib_lo_x16(w[tc][3]), nib_hi_x16(w[tc][3]), b[tc][mt][2], b[tc][mt][3],
                          ta[mt][0], ta[mt][1], ta[mt][2], ta[mt][3]);
      } else {
        mma_s8_m16n8k32_c(ta[mt], w[tc][0], w[tc][1], w[tc][2], w[tc][3], b[tc][mt][0],
                          b[tc][mt][1], 0, 0, 0, 0);
        mma_s8_m16n8k32_c(ta[mt], w[tc][4], w[tc][5], w[tc][6], w[tc][7], b[tc][mt][2],
                          b[tc][mt][3], ta[mt][0], ta[mt][1], ta[mt][2], ta[mt][3]);
      }
    }
    if (MODE == 2) {
#pragma unroll
      for (int mt = 0; mt < MT; mt++)
#pragma unroll
        for (int i = 0; i < 4; i++) gacc[mt][i] += ta[mt][i];
      continue;
    }
#pragma unroll
    for (int mt = 0; mt < MT; mt++)
#pragma unroll
      for (int i = 0; i < 4; i++) gacc[mt][i] = (t % GK == 0) ? ta[mt][i] : gacc[mt][i] + ta[mt][i];
    if ((t + 1) % GK != 0) continue;  // group not complete yet
    const int lg = t / GK;            // group index inside the stage
    if (MODE == 0) {
      float s0, s1;
      scale_pair(lg < 4 ? sc0 : sc1, (lg & 3) * 8, L.g8, s0, s1);
#pragma unroll
      for (int mt = 0; mt < MT; mt++)
#pragma unroll
        for (int i = 0; i < 4; i++)
          cf[mt][i] = __fmaf_rn(i2f_exact(gacc[mt][i] >> 4), i < 2 ? s0 : s1, cf[mt][i]);
    } else {
      const size_t gb = (size_t)(g0 + lg) * MT * 8;
      if (MODE == 3) {
        float s0, s1;
        scale_pair(lg < 4 ? sc0 : sc1, (lg & 3) * 8, L.g8, s0, s1);
        float *pf = reinterpret_cast<float *>(pub);
#pragma unroll
        for (int mt = 0; mt < MT; mt++)
#pragma unroll
          for (int i = 0; i < 4; i++)
            pf[(gb + mt * 8 + 2 * L.tig + (i & 1)) * (MT == 1 ? kPubRow : L.pr) + L.g8 +
               (i >= 2 ? 8 : 0)] =
                i2f_exact(gacc[mt][i] >> 4);
        if (L.tig == 0) {
          float *ps = reinterpret_cast<float *>(pub_sc) + (size_t)(g0 + lg) * 16;
          ps[L.g8] = s0;
          ps[L.g8 + 8] = s1;
        }
      } else {
#pragma unroll
        for (int mt = 0; mt < MT; mt++)
#pragma unroll
          for (int i = 0; i < 4; i++)
            pub[(gb + mt * 8 + 2 * L.tig + (i & 1)) * (MT == 1 ? kPubRow : L.pr) + L.g8 +
                (i >= 2 ? 8 : 0)] =
                gacc[mt][i] >> 4;
      }
    }
  }
  }
  if (MODE != 2)  // the stage ended on a group boundary: nothing carries over
#pragma unroll
    for (int mt = 0; mt < MT; mt++)
#pragma unroll
      for (int i = 0; i < 4; i++) gacc[mt][i] = 0;
}

// Any stage the fast path does not cover: a partial stage, activations read
// from global memory, or scale groups that straddle stages.  Scales are read
// from global memory here.  gacc carries a group across stage boundaries.
template <bool Q4, int MT, int GK, int MODE>
__device__ __forceinline__ void stage_generic(uint32_t st, uint32_t a_sm, const int8_t *abase,
                                              bool a_in, const Lane &L, int gt0, int nt, int gk,
                                              int nb, const GemvParams &p, uint32_t sc0,
                                              uint32_t sc1, float (&cf)[MT][4],
                                              int32_t (&gacc)[MT][4], int32_t *pub, int gbase,
                                              uint32_t *pub_sc) {
  constexpr int TB = Geo<Q4>::TB;
  for (int t = 0; t < nt; t++) {
    const int gt = gt0 + t;
    uint32_t w[Q4 ? 4 : 8];
#pragma unroll
    for (int q = 0; q < 4; q++) {
      if (Q4) {
        w[q] = lds32(st + t * TB + L.w_off + q * 128);
      } else {
        w[2 * q] = lds32(st + t * TB + L.w_off + q * 256);
        w[2 * q + 1] = lds32(st + t * TB + L.w_off + q * 256 + 32);
      }
    }
    uint32_t b[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; mt++) {
      if (a_in) {
        const uint4 v = lds128(a_sm + (gt * MT + mt) * 512 + L.a_off);
        b[mt][0] = v.x;
        b[mt][1] = v.y;
        b[mt][2] = v.z;
        b[mt][3] = v.w;
      } else {
        const int8_t *ar = abase + (size_t)gt * kATile + (mt * 8 + L.g8) * 64 + L.tig * 4;
        b[mt][0] = ld_shared_ro_u32(ar);
        b[mt][1] = ld_shared_ro_u32(ar + 16);
        b[mt][2] = ld_shared_ro_u32(ar + 32);
        b[mt][3] = ld_shared_ro_u32(ar + 48);
      }
    }
    int32_t ta[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; mt++) {
      if (Q4) {
        mma_s8_m16n8k32_c(ta[mt], nib_lo_x16(w[0]), nib_hi_x16(w[0]), nib_lo_x16(w[1]),
                          nib_hi_x16(w[1]), b[mt][0], b[mt][1], 0, 0, 0, 0);
        mma_s8_m16n8k32_c(ta[mt], nib_lo_x16(w[2]), nib_hi_x16(w[2]), nib_lo_x16(w[3]),
                          nib_hi_x16(w[3]), b[mt][2], b[mt][3], ta[mt][0], ta[mt][1], ta[mt][2],
                          ta[mt][3]);
      } else {
        mma_s8_m16n8k32_c(ta[mt], w[0], w[1], w[2], w[3], b[mt][0], b[mt][1], 0, 0, 0, 0);
        mma_s8_m16n8k32_c(ta[mt], w[4], w[5], w[6], w[7], b[mt][2], b[mt][3], ta[mt][0],
                          ta[mt][1], ta[mt][2], ta[mt][3]);
      }
    }
#pragma unroll
    for (int mt = 0; mt < MT; mt++)
#pragma unroll
      for (int i = 0; i < 4; i++) gacc[mt][i] += ta[mt][i];
    if (MODE == 2) continue;
    if ((gt + 1) % gk != 0) continue;
    const int g = gt / gk;
    const int lg = (gt - gt0) / gk;  // group index inside the stage (GK > 0 only)
    const bool exact_ok = GK || p.group <= kExactGroupMax;
    float s0 = 0.0f, s1 = 0.0f;
    if (MODE == 0 || MODE == 3) {
      if (GK) {  // groups tile the stage: the prefetched rows hold this group
        scale_pair(lg < 4 ? sc0 : sc1, (lg & 3) * 8, L.g8, s0, s1);
      } else {
        const __half *sr =
            reinterpret_cast<const __half *>(p.b_scale) + (size_t)g * p.N + nb * 16;
        s0 = __half2float(sr[L.g8]);
        s1 = __half2float(sr[L.g8 + 8]);
      }
    }
    if (MODE == 0) {
#pragma unroll
      for (int mt = 0; mt < MT; mt++)
#pragma unroll
        for (int i = 0; i < 4; i++)
          cf[mt][i] = __fmaf_rn(i2f_group(gacc[mt][i] >> 4, exact_ok), i < 2 ? s0 : s1, cf[mt][i]);
    } else {
      const size_t gb = (size_t)(g - gbase) * MT * 8;
      if (MODE == 3) {
        float *pf = reinterpret_cast<float *>(pub);
#pragma unroll
        for (int mt = 0; mt < MT; mt++)
#pragma unroll
          for (int i = 0; i < 4; i++)
            pf[(gb + mt * 8 + 2 * L.tig + (i & 1)) * (MT == 1 ? kPubRow : L.pr) + L.g8 +
               (i >= 2 ? 8 : 0)] =
                i2f_group(gacc[mt][i] >> 4, exact_ok);
        if (L.tig == 0) {
          float *ps = reinterpret_cast<float *>(pub_sc) + (size_t)(g - gbase) * 16;
          ps[L.g8] = s0;
          ps[L.g8 + 8] = s1;
        }
      } else {
#pragma unroll
        for (int mt = 0; mt < MT; mt++)
#pragma unroll
          for (int i = 0; i < 4; i++)
            pub[(gb + mt * 8 + 2 * L.tig + (i & 1)) * (MT == 1 ? kPubRow : L.pr) + L.g8 +
                (i >= 2 ? 8 : 0)] =
                gacc[mt][i] >> 4;
      }
    }
#pragma unroll
    for (int mt = 0; mt < MT; mt++)
#pragma unroll
      for (int i = 0; i < 4; i++) gacc[mt][i] = 0;
  }
}

template <bool Q4, int MT, int GK>
__global__ void __launch_bounds__(kMaxWarps * 32, 1)
    gemv_kernel(const GemvParams p, const GemvPlan pl) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int s_abort;
  __shared__ int s_slot;                  // fused gather: this call's buffer
  __shared__ unsigned long long s_uses;   // fused gather: calls that used it, this one included
  __shared__ float s_as[16];  // a_scale of the block's rows
  constexpr int TB = Geo<Q4>::TB;
  constexpr int T = Geo<Q4>::T;
  const bool raw = p.acc != nullptr;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, NW = blockDim.x >> 5;
  const int P = pl.parts, team = warp / P, part = warp % P, teams = NW / P;
  const int KB = p.K / kTileK;
  const int gk = Q4 ? (GK ? GK : p.group / kTileK) : KB;
  const int G = KB / gk;
  const int ptiles = KB / P;
  const int nch = (ptiles + T - 1) / T;
  const int S = pl.stages;
  // int4: part 0 of a team folds its groups in registers as they complete;
  // the other parts publish int32 group sums to the team's shared area (as
  // does every part for int32 output); int8: accumulate.
  const bool fold = Q4 && !raw && part == 0;
  const bool want_sc = Q4 && !raw;            // this warp needs its groups' scales
  const int gpub = (Q4 && !raw) ? G / P : 0;  // first group held in the shared area
  uint8_t *after_ring = smem + (size_t)NW * S * pl.stage_bytes;
  int32_t *xsum = reinterpret_cast<int32_t *>(after_ring + (size_t)team * pl.xchg_bytes);
  // part 0's running f32 outputs, handed to the team after the last group,
  // then the published groups' f32 scale rows (16 floats each)
  float *cpart = reinterpret_cast<float *>(xsum + (size_t)(G - gpub) * MT * 8 *
                                            (MT == 1 ? kPubRow : pl.pub_row));
  uint32_t *xscale = reinterpret_cast<uint32_t *>(cpart + MT * 128);
  uint32_t *pub_sc = (Q4 && !raw && P > 1) ? xscale : nullptr;
  uint32_t *a_sm = reinterpret_cast<uint32_t *>(after_ring + (size_t)teams * pl.xchg_bytes);
  uint64_t *bars = reinterpret_cast<uint64_t *>(reinterpret_cast<uint8_t *>(a_sm) + pl.a_bytes) +
                   warp * S;
  const uint32_t ring = tc::smem_u32(smem) + (uint32_t)(warp * S * pl.stage_bytes);
  const uint32_t a_sm_u = tc::smem_u32(a_sm);
  const int mb = blockIdx.y;
  const int8_t *abase = p.A + (size_t)mb * KB * kATile;

  Lane L;
  L.lane = lane;
  L.g8 = lane >> 2;
  L.tig = lane & 3;
  L.pr = MT == 1 ? kPubRow : pl.pub_row;
  L.w_off = Q4 ? (uint32_t)(L.tig * 32 + L.g8 * 4) : (uint32_t)(L.tig * 64 + L.g8 * 4);
  L.a_off = (uint32_t)(L.g8 * 64 + L.tig * 16);

  if (threadIdx.x == 0) s_abort = 0;
  if (lane == 0) {
    for (int s = 0; s < S; s++) tc::mbar_init(&bars[s], 1);
    tc::fence_mbar_init();
  }
  if (P > 1 && !Q4)
    for (int i = threadIdx.x; i < teams * MT * 128; i += blockDim.x)
      reinterpret_cast<int32_t *>(after_ring + (size_t)(i / (MT * 128)) * pl.xchg_bytes)
          [i % (MT * 128)] = 0;
  __syncthreads();
  pdl_launch_dependents();

  const int tstride = gridDim.x * teams;
  const int unit0 = blockIdx.x * teams + team;
  const int my_units = unit0 < pl.units ? (pl.units - unit0 + tstride - 1) / tstride : 0;
  const int items = my_units * nch;

  // issue cursor: (unit index, stage) of the next stage to fetch and its slot
  int iu = 0, ic = 0, islot = 0;
  auto issue = [&]() {
    const int nb = p.nb0 + unit0 + iu * tstride;
    const int gt0 = part * ptiles + ic * T;
    const int gt1 = min(gt0 + T, (part + 1) * ptiles);
    const uint32_t wbytes = (uint32_t)(gt1 - gt0) * TB;
    if (lane == 0) {
      tc::mbar_expect_tx(&bars[islot], wbytes);
      bulk_g2s(ring + islot * pl.stage_bytes, p.B + ((size_t)nb * KB + gt0) * TB, wbytes,
               &bars[islot]);
    }
    if (++ic == nch) {
      ic = 0;
      iu++;
    }
    if (++islot == S) islot = 0;
  };
  // scale cursor (int4 fold): lane l holds word l%8 of the stage's group rows
  // glo + l/8 and glo + 4 + l/8, fetched two stages ahead
  int su = 0, sch = 0;
  auto scale_fetch = [&](uint32_t &r0, uint32_t &r1) {
    r0 = r1 = 0;
    if (su >= my_units) return;
    const int nb = p.nb0 + unit0 + su * tstride;
    const int gt0 = part * ptiles + sch * T;
    const int gt1 = min(gt0 + T, (part + 1) * ptiles);
    const int glo = gt0 / gk, ng = gt1 / gk - glo;
    const uint8_t *row = reinterpret_cast<const uint8_t *>(p.b_scale) +
                         ((size_t)glo * p.N + (size_t)nb * 16) * 2 + (lane & 7) * 4;
    const int r = lane >> 3;
    if (r < ng) r0 = ldg_stream_u32(row + (size_t)r * p.N * 2);
    if (r + 4 < ng) r1 = ldg_stream_u32(row + (size_t)(r + 4) * p.N * 2);
    if (++sch == nch) {
      sch = 0;
      su++;
    }
  };

  // Stages requested before griddepcontrol.wait overlap a predecessor that is
  // still running; the rest go out after the activation loads, so those loads
  // do not queue behind a full weight stream (they gate every MMA).
  const int prologue = items < S ? items : S;
  const int pre = prologue < pl.pre_stages ? prologue : pl.pre_stages;
  for (int it = 0; it < pre; it++) issue();
  // the next launch's weights follow this launch's own stage requests into
  // the memory system, so HBM keeps streaming across the kernel boundary
  if (blockIdx.y == 0 && warp == NW - 1 && (p.warm_bytes[0] | p.warm_bytes[1])) warm_next(p, lane);
  uint32_t sc_a0 = 0, sc_a1 = 0, sc_b0 = 0, sc_b1 = 0;  // stages it and it+1
  if (want_sc && GK) {
    scale_fetch(sc_a0, sc_a1);
    scale_fetch(sc_b0, sc_b1);
  }
  pdl_wait();  // activations and outputs are ordered after earlier kernels
  if (p.g.world > 0 && threadIdx.x == 0) {
    // this call's slot from the rank's completed-call counter (the previous
    // call finished before griddepcontrol.wait returned)
    const unsigned long long c = ld_acquire_sys(p.g.sig[p.g.rank] + 6);
    s_slot = (int)(c & 1);
    s_uses = (c >> 1) + 1;
    if (blockIdx.x == 0 && blockIdx.y == 0) {
      p.g.sig[p.g.rank][8] = tc::globaltimer_ns();
      // everything before this call on this stream is complete, including the
      // readers of this slot's previous contents: tell every rank it may write.
      // Each warp checks that every rank did the same just before its first
      // push, so the weight stream and the first units do not wait for it.
      for (int q = 0; q < p.g.world; q++) atomicAdd_system(p.g.sig[q] + 2 + s_slot, 1ull);
    }
  }

  // the row block's activation scales ride in the same round trip as the
  // activation staging (one L2 latency after griddepcontrol.wait, not two)
  const bool load_as = !raw && threadIdx.x < MT * 8;
  float as_v = 0.0f;
  if (load_as) {
    const int m = mb * 16 + threadIdx.x;
    as_v = m < p.M ? p.a_scale[m] : 0.0f;
  }
  if (pl.a_bytes) {  // stage this row block's activations, B-fragment order
    // 16-byte pieces: piece c of a 64-byte row holds k-quads 4c..4c+3, which
    // land at word positions j*4 + c.  Loads go out in independent batches.
    constexpr int kBatchLd = 8;
    const int pieces = KB * MT * 8 * 4;
    const int step = kBatchLd * blockDim.x;
    for (int b0 = 0; b0 < pieces; b0 += step) {  // the same trip count in every thread
      const int base = b0 + threadIdx.x;
      uint4 v[kBatchLd];
#pragma unroll
      for (int u = 0; u < kBatchLd; u++) {
        const int i = base + u * blockDim.x;
        if (i < pieces) {
          const int c = i & 3, row = (i >> 2) % (MT * 8), tile = (i >> 2) / (MT * 8);
          v[u] = *reinterpret_cast<const uint4 *>(abase + (size_t)tile * kATile + row * 64 + c * 16);
        }
      }
      if (b0 == 0)  // the first batch is in flight: now the rest of the weight prologue
        for (int it = pre; it < prologue; it++) issue();
#pragma unroll
      for (int u = 0; u < kBatchLd; u++) {
        const int i = base + u * blockDim.x;
        if (i < pieces) {
          const int c = i & 3, rowg = i >> 2;  // rowg = tile * MT*8 + row
          uint32_t *d = a_sm + (rowg << 4) + c;
          d[0] = v[u].x;
          d[4] = v[u].y;
          d[8] = v[u].z;
          d[12] = v[u].w;
        }
      }
    }
  } else {
    for (int it = pre; it < prologue; it++) issue();
  }
  if (load_as) s_as[threadIdx.x] = as_v;
  if (pl.a_bytes || !raw || p.g.world > 0) __syncthreads();
  const int gslot = p.g.world > 0 ? s_slot : 0;
  const unsigned long long guses = p.g.world > 0 ? s_uses : 0;
  float *const Cout = p.C + (size_t)gslot * p.g.slot_floats;  // this call's output buffer
  bool pushed = false;  // this warp has checked that every peer's slot is free

  float cf[MT][4];
  int32_t gacc[MT][4];
  int cu = 0, cc = 0, cslot = 0;
  uint32_t cphase = 0;
  for (int it = 0; it < items; it++) {
    const int nb = p.nb0 + unit0 + cu * tstride;
    const int gt0 = part * ptiles + cc * T;
    const int nt = min(T, (part + 1) * ptiles - gt0);
    if (cc == 0) {
#pragma unroll
      for (int mt = 0; mt < MT; mt++)
#pragma unroll
        for (int i = 0; i < 4; i++) {
          cf[mt][i] = 0.0f;
          gacc[mt][i] = 0;
        }
    }
    const uint32_t sc0 = sc_a0, sc1 = sc_a1;
    if (want_sc && GK) {  // rotate the two-ahead scale prefetch
      sc_a0 = sc_b0;
      sc_a1 = sc_b1;
      scale_fetch(sc_b0, sc_b1);
    }
    bool ok = !*reinterpret_cast<volatile int *>(&s_abort) && tc::mbar_wait(&bars[cslot], cphase);
    ok = __all_sync(0xffffffffu, ok);
    if (!ok) {
      s_abort = 1;
      if (lane == 0 && p.err) atomicExch(p.err, 1);
    }
    const uint32_t st = ring + cslot * pl.stage_bytes;
    if (ok) {
      const bool fast = GK && pl.a_bytes && nt == T;
      const uint32_t ab = a_sm_u + (uint32_t)(gt0 * MT * 512);
      const bool a_in = pl.a_bytes != 0;
      if (!Q4) {
        if (fast) stage_full<Q4, MT, 1, T, 2>(st, ab, L, 0, 0, 0, cf, gacc, nullptr, nullptr);
        else
          stage_generic<Q4, MT, 0, 2>(st, a_sm_u, abase, a_in, L, gt0, nt, gk, nb, p, 0, 0, cf,
                                      gacc, nullptr, 0, nullptr);
      } else if (fold) {
        if (fast)
          stage_full<Q4, MT, GK ? GK : 1, T, 0>(st, ab, L, 0, sc0, sc1, cf, gacc, nullptr,
                                                nullptr);
        else
          stage_generic<Q4, MT, GK, 0>(st, a_sm_u, abase, a_in, L, gt0, nt, gk, nb, p, sc0, sc1,
                                       cf, gacc, nullptr, 0, nullptr);
      } else if (raw) {
        if (fast)
          stage_full<Q4, MT, GK ? GK : 1, T, 1>(st, ab, L, gt0 / gk - gpub, sc0, sc1, cf, gacc,
                                                xsum, nullptr);
        else
          stage_generic<Q4, MT, GK, 1>(st, a_sm_u, abase, a_in, L, gt0, nt, gk, nb, p, sc0, sc1,
                                       cf, gacc, xsum, gpub, nullptr);
      } else {
        if (fast)
          stage_full<Q4, MT, GK ? GK : 1, T, 3>(st, ab, L, gt0 / gk - gpub, sc0, sc1, cf, gacc,
                                                xsum, pub_sc);
        else
          stage_generic<Q4, MT, GK, 3>(st, a_sm_u, abase, a_in, L, gt0, nt, gk, nb, p, sc0, sc1,
                                       cf, gacc, xsum, gpub, pub_sc);
      }
    }
    __syncwarp();
    fence_proxy_async_smem();
    if (ok && it + S < items) issue();
    if (++cslot == S) {
      cslot = 0;
      cphase ^= 1u;
    }
    const bool unit_done = (cc == nch - 1);
    if (++cc == nch) {
      cc = 0;
      cu++;
    }
    if (!unit_done) continue;

    // ---- this warp's part of unit nb is done
    if (P == 1) {
      if (!ok) continue;
      if (Q4 && raw) {  // the warp's published group sums -> acc[m][g][n]
        __syncwarp();
        for (int o = lane; o < G * MT * 128; o += 32) {
          const int g = o / (MT * 128), r = o % (MT * 128), ml = r >> 4, nl = r & 15;
          const int m = mb * 16 + ml;
          if (m < p.M)
            p.acc[((size_t)m * G + g) * p.N + nb * 16 + nl] =
                xsum[((size_t)g * MT * 8 + ml) * L.pr + nl];
        }
        __syncwarp();
        continue;
      }
#pragma unroll
      for (int mt = 0; mt < MT; mt++)
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const int m = mb * 16 + mt * 8 + 2 * L.tig + (i & 1);
          const int n = nb * 16 + L.g8 + (i >= 2 ? 8 : 0);
          if (m >= p.M) continue;
          if (raw) {
            p.acc[(size_t)m * p.N + n] = gacc[mt][i];
          } else if (Q4) {
            Cout[(size_t)m * p.ldc + (n - p.c_col0)] = __fmul_rn(cf[mt][i], s_as[m - mb * 16]);
          } else {
            const float bs = reinterpret_cast<const float *>(p.b_scale)[n];
            Cout[(size_t)m * p.ldc + (n - p.c_col0)] =
                __fmul_rn(__int2float_rn(gacc[mt][i]), __fmul_rn(bs, s_as[m - mb * 16]));
          }
        }
      if (p.g.world > 0 && !*reinterpret_cast<volatile int *>(&s_abort)) {
        if (!pushed && !(pushed = peers_free(p, gslot, guses, lane))) {
          s_abort = 1;
          if (lane == 0 && p.err) atomicExch(p.err, 3);
          continue;
        }
        __syncwarp();  // this warp's stores of the unit are visible to its lanes
#pragma unroll
        for (int r0 = 0; r0 < MT * 8; r0 += 8) push_rows(p, Cout, nb, mb * 16 + r0, lane);
      }
      continue;
    }
    if (!Q4) {  // int8 split K: add the int32 partials
#pragma unroll
      for (int mt = 0; mt < MT; mt++)
#pragma unroll
        for (int i = 0; i < 4; i++)
          atomicAdd(&xsum[(mt * 8 + 2 * L.tig + (i & 1)) * 16 + L.g8 + (i >= 2 ? 8 : 0)],
                    gacc[mt][i]);
    }
    if (Q4 && !raw && part == 0 && ok) {  // hand the chain over to the team
#pragma unroll
      for (int mt = 0; mt < MT; mt++)
#pragma unroll
        for (int i = 0; i < 4; i++)
          cpart[(mt * 8 + 2 * L.tig + (i & 1)) * 16 + L.g8 + (i >= 2 ? 8 : 0)] = cf[mt][i];
    }
    team_sync(team, P * 32);
    for (int o = part * 32 + lane; o < MT * 128; o += P * 32) {
      const int ml = o >> 4, nl = o & 15;
      const int m = mb * 16 + ml, n = nb * 16 + nl;
      if (Q4) {
        if (m >= p.M) continue;
        if (raw) {
          for (int g = 0; g < G; g++)
            p.acc[((size_t)m * G + g) * p.N + n] = xsum[((size_t)g * MT * 8 + ml) * L.pr + nl];
          continue;
        }
        // continue part 0's chain through the published groups, in order
        const float *xf = reinterpret_cast<const float *>(xsum) + ml * L.pr + nl;
        const float *xs = reinterpret_cast<const float *>(xscale) + nl;
        float c = cpart[o];
        const int ng = G - gpub;
        const size_t gstride = (size_t)MT * 8 * L.pr;
#pragma unroll 8
        for (int g = 0; g < ng; g++) c = __fmaf_rn(xf[g * gstride], xs[g * 16], c);
        Cout[(size_t)m * p.ldc + (n - p.c_col0)] = __fmul_rn(c, s_as[ml]);
      } else {
        const int32_t v = xsum[ml * 16 + nl];
        xsum[ml * 16 + nl] = 0;
        if (m >= p.M) continue;
        if (raw) {
          p.acc[(size_t)m * p.N + n] = v;
        } else {
          const float bs = reinterpret_cast<const float *>(p.b_scale)[n];
          Cout[(size_t)m * p.ldc + (n - p.c_col0)] =
              __fmul_rn(__int2float_rn(v), __fmul_rn(bs, s_as[ml]));
        }
      }
    }
    team_sync(team, P * 32);
    if (p.g.world > 0 && part < MT && !*reinterpret_cast<volatile int *>(&s_abort)) {
      if (!pushed && !(pushed = peers_free(p, gslot, guses, lane))) {
        s_abort = 1;
        if (lane == 0 && p.err) atomicExch(p.err, 3);
      } else {
        push_rows(p, Cout, nb, mb * 16 + part * 8, lane);
      }
    }
  }

  if (p.g.world > 0) {
    // ---- fused all-gather: every unit of this CTA has been pushed; publish
    // the pushes, count this CTA, and let the rank's last CTA signal every
    // rank and wait until its own buffer holds all ranks' columns.
    const GatherParams &g = p.g;
    const unsigned long long need = (unsigned long long)g.world * guses;
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
      const unsigned long long done = atomicAdd(g.sig[g.rank] + 4 + gslot, 1ull) + 1;
      if (done == guses * gridDim.x * gridDim.y) {  // this rank's last CTA
        __threadfence_system();
        g.sig[g.rank][9] = tc::globaltimer_ns();
        for (int q = 0; q < g.world; q++) atomicAdd_system(g.sig[q] + gslot, 1ull);
        // the call completes when every rank's columns are in this buffer
        if (!spin_until_geq(g.sig[g.rank] + gslot, need) && p.err) atomicExch(p.err, 3);
        g.sig[g.rank][10] = tc::globaltimer_ns();
        // the next call on this rank uses the other buffer (it reads this
        // counter after griddepcontrol.wait, i.e. after this kernel completed)
        __threadfence_system();
        atomicAdd(g.sig[g.rank] + 6, 1ull);
      }
    }
  }
}

template <bool Q4, int MT, int GK>
cudaError_t launch_t(const GemvParams &p, const GemvPlan &pl, dim3 grid, bool pdl,
                     cudaStream_t st) {
  auto kern = gemv_kernel<Q4, MT, GK>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)pl.smem_bytes);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(pl.warps * 32);
  cfg.dynamicSmemBytes = pl.smem_bytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, p, pl);
}

template <bool Q4, int MT>
cudaError_t launch_gk(const GemvParams &p, const GemvPlan &pl, dim3 grid, bool pdl,
                      cudaStream_t st) {
  if constexpr (!Q4) {
    return launch_t<Q4, MT, 1>(p, pl, grid, pdl, st);
  } else {
    switch (p.group / kTileK) {  // groups that tile a stage exactly
      case 1: return launch_t<Q4, MT, 1>(p, pl, grid, pdl, st);
      case 2: return launch_t<Q4, MT, 2>(p, pl, grid, pdl, st);
      case 4: return launch_t<Q4, MT, 4>(p, pl, grid, pdl, st);
      case 8: return launch_t<Q4, MT, 8>(p, pl, grid, pdl, st);
      default: return launch_t<Q4, MT, 0>(p, pl, grid, pdl, st);  // groups spanning stages
    }
  }
}

}  // namespace

// Pick the warp team size, warps per CTA, ring depth, activation staging and
// grid for a launch.
GemvPlan plan_gemv(const GemvParams &p, int nblocks, bool q4, int num_sms, size_t smem_limit) {
  GemvPlan pl{};
  const int MT = p.M <= 8 ? 1 : 2;
  const int KB = p.K / kTileK, gk = q4 ? p.group / kTileK : KB, G = KB / gk;
  const int TB = q4 ? kQ4Tile : kQ8Tile;
  const int T = q4 ? Geo<true>::T : Geo<false>::T;
  const bool raw = p.acc != nullptr;
  pl.warps = kMaxWarps;
  pl.units = nblocks;
  pl.parts = 1;
  pl.ctas_per_sm = 1;
  pl.chunk_tiles = T;
  // team size: enough (unit, part) pairs to give every warp of the grid work,
  // but every part keeps at least one full ring stage of tiles (the unrolled
  // stage path; thinner parts only add warps that finish their few tiles at
  // the same moment and a longer serial fold)
  int Pmax = 1;
  const int want = num_sms * kMaxWarps;
  while (Pmax < kMaxWarps && (long)nblocks * Pmax * 2 <= want) {
    const int P2 = Pmax * 2;
    const bool parts_ok = (q4 ? (G % P2 == 0) : (KB % P2 == 0)) && KB / P2 >= T;
    if (!parts_ok) break;
    Pmax = P2;
  }
  pl.stage_bytes = (T * TB + 127) / 128 * 128;
  const size_t a_bytes = (size_t)KB * MT * 8 * 64;
  // Activations in shared memory first (reading them per tile from global
  // memory exposes L2 latency on every tile), then the largest team size whose
  // exchange area still leaves a useful ring.  Warps per CTA: enough to cover
  // every (unit, part) pair across all SMs, at most kMaxWarps, a multiple of
  // the team size.  Then the deepest ring that fits.
  // One search per exchange row stride; the padded stride wins unless the
  // dense one keeps the activations staged or more split-K parts.
  auto search = [&](int pub_row, GemvPlan &out) {
  bool found = false;
  for (int with_a = 1; with_a >= 0 && !found; with_a--) {
  for (int P = Pmax; P >= 1 && !found; P /= 2) {
    const long pairs = (long)nblocks * P;
    int want_warps = (int)((pairs + num_sms - 1) / num_sms);
    want_warps = (want_warps + P - 1) / P * P;
    if (want_warps > kMaxWarps) want_warps = kMaxWarps;
    if (want_warps < P) want_warps = P;
    size_t xchg = 0;
    const size_t grp = (size_t)MT * 8 * pub_row * 4;  // one group's published values
    if (q4 && raw) xchg = (size_t)G * grp;             // every group's int32 sum
    else if (q4 && P > 1)  // groups of parts 1..P-1 with their f32 scale rows, part 0's chain
      xchg = (size_t)(G - G / P) * (grp + 64) + (size_t)MT * 128 * 4;
    else if (P > 1) xchg = (size_t)MT * 128 * 4;  // int8 partials
    const int xchg_bytes = (int)((xchg + 127) / 128 * 128);
    // fewer warps per CTA when the exchange areas would not fit otherwise
    for (int warps = want_warps; warps >= P && !found; warps -= P) {
      const int teams = warps / P;
      const size_t bars_w = (size_t)warps * 8 * 8;
      {
        const size_t fixed = (size_t)teams * xchg_bytes + (with_a ? a_bytes : 0) + bars_w;
        for (int S = 6; S >= 2; S--) {
          const size_t total = fixed + (size_t)warps * S * pl.stage_bytes;
          if (total <= smem_limit) {
            out.warps = warps;
            out.parts = P;
            out.xchg_bytes = xchg_bytes;
            out.stages = S;
            out.pre_stages = 1;
            out.pub_row = pub_row;
            out.a_bytes = with_a ? (int)a_bytes : 0;
            out.smem_bytes = total;
            found = true;
            break;
          }
        }
      }
    }
  }
  }
  return found;
  };
  GemvPlan dense = pl;
  bool found = search(kPubRow, pl);
  if (MT == 2 && search(kPubRowDense, dense) &&
      (!found || (dense.a_bytes && !pl.a_bytes) ||
       ((dense.a_bytes != 0) == (pl.a_bytes != 0) && dense.parts > pl.parts))) {
    pl = dense;
    found = true;
  }
  if (!found) {  // caller reports the failure; stages = 0 marks the plan unusable
    pl.stages = 0;
    pl.smem_bytes = smem_limit + 1;
  }
  const int teams = pl.warps / pl.parts;
  const int ctas_needed = (nblocks + teams - 1) / teams;
  pl.grid_x = ctas_needed < num_sms ? ctas_needed : num_sms;
  return pl;
}

cudaError_t launch_gemv(const GemvParams &p, int nblocks, bool q4, bool pdl, int num_sms,
                        size_t smem_limit, cudaStream_t st) {
  if (nblocks <= 0 || p.M <= 0) return cudaSuccess;
  const GemvPlan pl = plan_gemv(p, nblocks, q4, num_sms, smem_limit);
  if (pl.stages < 2 || pl.warps < 1 || pl.smem_bytes > smem_limit)
    return cudaErrorInvalidConfiguration;
  const dim3 grid(pl.grid_x, (p.M + 15) / 16);
  const bool mt1 = p.M <= 8;
  if (q4)
    return mt1 ? launch_gk<true, 1>(p, pl, grid, pdl, st) : launch_gk<true, 2>(p, pl, grid, pdl, st);
  return mt1 ? launch_gk<false, 1>(p, pl, grid, pdl, st) : launch_gk<false, 2>(p, pl, grid, pdl, st);
}

}  // namespace fgm
