// A decode step's projections as one persistent launch: a work list of
// quantised decode GEMMs (and the activation preps that feed them) whose
// weight stream never stops at an item boundary.
//
// Reference: each GEMM item is fgm_gemm_q4g / fgm_gemm_q8c (amx_gemm.c:333-475,
// vnni_gemm.c:224-322) on the .fgm tile layout, each prep item one row of
// fgm_prep_rows (ops.c:293-314: FWHT, fgm_quant_act, pack), i.e. what
// fgm-core's Gemm::run (forward.rs:128-158) does per projection; the list is
// the sequence of Gemm::run calls of a decode step.
//
// Why one launch
// --------------
// A decode GEMM at M <= 16 moves 0.5-18 MB of weights; as its own launch it
// pays a few microseconds of fixed latency (CTA start, activation staging,
// the drain of the last stages) that the weight stream cannot hide.  Here
// every consumer warp streams the weight tiles of ITS units of ALL items
// through its own shared-memory ring, so the ring of the next item fills
// while the current one finishes, and an item's inputs are ordered by
// completion counters instead of kernel boundaries.
//
// Schedule (built on the host, worklist_create)
// ---------------------------------------------
// Items are levelled by their dependencies (an item's level is one more than
// its deepest dependency).  Levels run in order; inside a level the items'
// units -- 16-column n-blocks of a GEMM over all of K, or single rows of a
// prep -- are spread over all CTAs: an item whose units cost more than twice
// the level's cheapest gets CTAs of its own (about half of each one's
// share), the other GEMM units fill every CTA's remaining share in
// contiguous ranges (biggest item first), prep rows go round-robin.  A
// CTA's share is a list of segments (item, unit range), its large units
// first.  The preps that depend on nothing are prepared at the start of the
// run by the CTAs their rows are dealt to (all consumer warps of a CTA
// together).  Consumer warps take a CTA's units from a shared counter in
// list order, so the lowest unfinished item can always progress: the kernel
// cannot deadlock while all CTAs are resident (grid = one CTA per SM).
//
// CTA roles
// ---------
// Warp 0 (producer) stages each GEMM segment's activations: it waits for the
// item's dependencies (counters in global memory, acquire loads), then one
// 3-D TMA box brings the segment's packed rows [tiles][rows][64 B] into a
// region of the activation ring (first fit) with the 64-byte swizzle, so the
// consumers' B-fragment loads (k-quads t, 4+t, 8+t, 12+t of row g) hit 32
// distinct banks.  Warps 1..W (consumers, W <= 15) each own a ring of
// 4352-byte stages (4 KB of weights: 8 int4 or 4 int8 tiles by one bulk
// copy, plus the int4 scale rows of its groups by one 2-D TMA box), refilled
// as soon as a stage is consumed, across unit and item boundaries.  The
// arithmetic per stage is the decode kernel's (gemv.cu): mma.sync m16n8k32
// s8 with the weights as the A operand read straight from the tile layout,
// int32 group sums, and the fold C = fmaf((float)acc_g, s_g, C) over
// ascending groups, then * a_scale (amx_gemm.c:103-113, :365-371); int8:
// (float)acc * (b_scale * a_scale) (amx_gemm.c:399).  Bit-identical to the
// per-call kernels.
//
// Waits and failures
// ------------------
// Every wait (mbarriers, dependency counters) gives up after 2 s or as soon
// as another warp has raised the list's abort word; the kernel then raises
// the device error word, waits (bounded) for its own copies in flight and
// returns.  The last CTA to finish resets the counters for the next launch.

#include <cuda.h>

#include <algorithm>
#include <functional>
#include <cstdlib>
#include <type_traits>
#include <cstring>
#include <vector>

#include "fgm_common.cuh"
#include "fgm_internal.h"
#include "stream_ptx.cuh"
#include "tc_ptx.cuh"

namespace fgm {

namespace {

using namespace stream;

constexpr int kWlStageW = 4096;    // weight bytes per ring stage (8 int4 or 4 int8 tiles)
constexpr int kWlStageS = 256;     // int4 scale rows of the stage (up to 8 groups x 32 bytes)
constexpr int kWlStage = kWlStageW + kWlStageS;  // bytes per ring stage
constexpr int kWlMaxStages = 8;
constexpr int kWlASlots = 4;       // GEMM segments whose activations can be staged at once
constexpr uint64_t kWlLimitNs = 2000000000ull;

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned *a) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
  return v;
}

__device__ __forceinline__ int ld_volatile(const int *a) {
  return *reinterpret_cast<const volatile int *>(a);
}

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Raise the abort word (list) and the device error word.
__device__ __forceinline__ void wl_fail(const WlParams &p, int code) {
  atomicExch(p.abort, 1);
  if (p.err) atomicExch(p.err, code);
}

// mbarrier phase wait, bounded in time and abandoned when the list aborts.
// The abort word (a global load, an L2 round trip) is read only once a wait
// has lasted 20 us: a normal wait then reacts as soon as the phase completes.
__device__ __forceinline__ bool wl_wait(uint64_t *bar, uint32_t parity, const WlParams &p) {
  if (tc::mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = tc::globaltimer_ns();
  while (!tc::mbar_try_wait(bar, parity)) {
    const uint64_t dt = tc::globaltimer_ns() - t0;
    if (dt > 20000 && ld_volatile(p.abort)) return false;  // another warp gave up
    if (dt > kWlLimitNs) return false;
  }
  return true;
}

// Wait until every unit of item `dep` has completed (counter == units).
__device__ __forceinline__ bool wl_wait_item(const WlParams &p, int dep) {
  if (dep < 0) return true;
  const unsigned need = (unsigned)p.items[dep].units;
  if (ld_acquire_gpu(p.done + dep) >= need) return true;
  const uint64_t t0 = tc::globaltimer_ns();
  while (ld_acquire_gpu(p.done + dep) < need) {
    if (ld_volatile(p.abort)) return false;
    if (tc::globaltimer_ns() - t0 > kWlLimitNs) return false;
    __nanosleep(64);
  }
  return true;
}

// Publish `n` completed units of item `it` (after this warp's stores).
__device__ __forceinline__ void wl_signal(const WlParams &p, int it, unsigned n, int lane) {
  fence_proxy_async_global();  // the next reader may be a TMA load (async proxy)
  __syncwarp();
  if (lane == 0) {
    __threadfence();
    atomicAdd(p.done + it, n);
  }
}

// 2-D TMA load to a shared-memory address given as a 32-bit shared pointer.
__device__ __forceinline__ void tma_load_2d_u32(uint32_t dst, const void *tmap, uint64_t *bar,
                                                int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(tmap), "r"(tc::smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ uint32_t lds16(uint32_t a) {
  unsigned short v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
  return v;
}

// Per-lane fragment constants.
struct WlLane {
  int g8, tig;
  uint32_t w4_off, w8_off;  // weight word (row tig, column g8) in an int4 / int8 tile
  uint32_t a_off[4];        // k-quad chunk c of activation row g8 in a swizzled 64-byte row
};

__device__ __forceinline__ WlLane make_lane(int lane) {
  WlLane L;
  L.g8 = lane >> 2;
  L.tig = lane & 3;
  L.w4_off = (uint32_t)(L.tig * 32 + L.g8 * 4);
  L.w8_off = (uint32_t)(L.tig * 64 + L.g8 * 4);
#pragma unroll
  for (int c = 0; c < 4; c++)
    L.a_off[c] = (uint32_t)(L.g8 * 64 + ((c ^ ((L.g8 >> 1) & 3)) << 4) + L.tig * 4);
  return L;
}

// B fragments (activations) of tile t, row block mt: k-quads tig, 4+tig,
// 8+tig, 12+tig of row mt*8 + g8.
template <int MT>
__device__ __forceinline__ void load_b(uint32_t ab, int t, int mt, const WlLane &L,
                                       uint32_t (&b)[4]) {
  const uint32_t base = ab + (uint32_t)(t * MT * 512 + mt * 512);
#pragma unroll
  for (int c = 0; c < 4; c++) b[c] = lds32(base + L.a_off[c]);
}

// One 4 KB stage of an int4 unit: 8 tiles, scale groups of GK tiles folded
// into cf as they complete (the stage starts on a group boundary).
template <int MT, int GK>
__device__ __forceinline__ void q4_stage(uint32_t st, uint32_t ab, const WlLane &L,
                                         float2 (&cf)[MT][2]) {
  constexpr int CH = MT == 1 ? 4 : 2;  // tiles whose operands load together
  int32_t gacc[MT][4];
#pragma unroll
  for (int t0 = 0; t0 < 8; t0 += CH) {
    uint32_t w[CH][4];
    uint32_t b[CH][MT][4];
#pragma unroll
    for (int tc = 0; tc < CH; tc++) {
      const int t = t0 + tc;
#pragma unroll
      for (int q = 0; q < 4; q++) w[tc][q] = lds32(st + t * 512 + L.w4_off + q * 128);
#pragma unroll
      for (int mt = 0; mt < MT; mt++) load_b<MT>(ab, t, mt, L, b[tc][mt]);
    }
#pragma unroll
    for (int tc = 0; tc < CH; tc++) {
      const int t = t0 + tc;
      int32_t ta[MT][4];
#pragma unroll
      for (int mt = 0; mt < MT; mt++) {
        mma_s8_m16n8k32_c(ta[mt], nib_lo_x16(w[tc][0]), nib_hi_x16(w[tc][0]),
                          nib_lo_x16(w[tc][1]), nib_hi_x16(w[tc][1]), b[tc][mt][0], b[tc][mt][1],
                          0, 0, 0, 0);
        mma_s8_m16n8k32_c(ta[mt], nib_lo_x16(w[tc][2]), nib_hi_x16(w[tc][2]),
                          nib_lo_x16(w[tc][3]), nib_hi_x16(w[tc][3]), b[tc][mt][2], b[tc][mt][3],
                          ta[mt][0], ta[mt][1], ta[mt][2], ta[mt][3]);
      }
#pragma unroll
      for (int mt = 0; mt < MT; mt++)
#pragma unroll
        for (int i = 0; i < 4; i++)
          gacc[mt][i] = (t % GK == 0) ? ta[mt][i] : gacc[mt][i] + ta[mt][i];
      if ((t + 1) % GK != 0) continue;
      const int lg = t / GK;  // group inside the stage: its f16 scale row follows the tiles
      const uint32_t srow = st + kWlStageW + lg * 32 + L.g8 * 2;
      const float s0 = f16_to_f32(lds16(srow)), s1 = f16_to_f32(lds16(srow + 16));
      const float2 sp0 = make_float2(s0, s0), sp1 = make_float2(s1, s1);
#pragma unroll
      for (int mt = 0; mt < MT; mt++) {
        // the group sums as exact floats, two per instruction, then the
        // reference's fma into the running sums (each lane rounded alone)
        float2 f01, f23;
        if (GK <= 4) {
          // gacc = 16 x the group sum, |sum| <= 2^18 for groups up to 256:
          // added to the bit pattern of 1.5 * 2^19 (ulp 1/16) it gives
          // 1.5 * 2^19 + sum exactly, no shift needed
          f01 = __fadd2_rn(make_float2(__int_as_float(gacc[mt][0] + 0x49400000),
                                       __int_as_float(gacc[mt][1] + 0x49400000)),
                           make_float2(-786432.0f, -786432.0f));
          f23 = __fadd2_rn(make_float2(__int_as_float(gacc[mt][2] + 0x49400000),
                                       __int_as_float(gacc[mt][3] + 0x49400000)),
                           make_float2(-786432.0f, -786432.0f));
        } else {
          f01 = make_float2(i2f_exact(gacc[mt][0] >> 4), i2f_exact(gacc[mt][1] >> 4));
          f23 = make_float2(i2f_exact(gacc[mt][2] >> 4), i2f_exact(gacc[mt][3] >> 4));
        }
        cf[mt][0] = __ffma2_rn(f01, sp0, cf[mt][0]);
        cf[mt][1] = __ffma2_rn(f23, sp1, cf[mt][1]);
      }
    }
  }
}

// One 4 KB stage of an int8 unit: 4 tiles accumulated in int32.
template <int MT>
__device__ __forceinline__ void q8_stage(uint32_t st, uint32_t ab, const WlLane &L,
                                         int32_t (&acc)[MT][4]) {
#pragma unroll
  for (int t = 0; t < 4; t++) {
    uint32_t w[8];
#pragma unroll
    for (int q = 0; q < 4; q++) {
      w[2 * q] = lds32(st + t * 1024 + L.w8_off + q * 256);
      w[2 * q + 1] = lds32(st + t * 1024 + L.w8_off + q * 256 + 32);
    }
#pragma unroll
    for (int mt = 0; mt < MT; mt++) {
      uint32_t b[4];
      load_b<MT>(ab, t, mt, L, b);
      int32_t ta[4];
      mma_s8_m16n8k32_c(ta, w[0], w[1], w[2], w[3], b[0], b[1], 0, 0, 0, 0);
      mma_s8_m16n8k32_c(ta, w[4], w[5], w[6], w[7], b[2], b[3], ta[0], ta[1], ta[2], ta[3]);
#pragma unroll
      for (int i = 0; i < 4; i++) acc[mt][i] += ta[i];
    }
  }
}

// ------------------------------------------------------------------ prep row
__device__ __forceinline__ float bfly(float own, int lm, bool hi) {
  const float other = __shfl_xor_sync(0xffffffffu, own, lm);
  return hi ? __fsub_rn(other, own) : __fadd_rn(own, other);
}

// Normalised FWHT (ops.c:153-175) of the hsz-blocks (hsz <= 128) of one
// 128-value chunk held as lane l's values 4l..4l+3: the reference's stage
// order and pairing, then 1/sqrt(hsz) for blocks of 16 or more (its vector
// loop leaves smaller blocks unscaled).
__device__ __forceinline__ float4 fwht128(float4 u, int hsz, int lane) {
  if (hsz > 1) {
    u = make_float4(__fadd_rn(u.x, u.y), __fsub_rn(u.x, u.y), __fadd_rn(u.z, u.w),
                    __fsub_rn(u.z, u.w));
  }
  if (hsz > 2) {
    u = make_float4(__fadd_rn(u.x, u.z), __fadd_rn(u.y, u.w), __fsub_rn(u.x, u.z),
                    __fsub_rn(u.y, u.w));
  }
  for (int len = 4; len < hsz; len <<= 1) {
    const int lm = len >> 2;
    const bool hi = (lane & lm) != 0;
    u.x = bfly(u.x, lm, hi);
    u.y = bfly(u.y, lm, hi);
    u.z = bfly(u.z, lm, hi);
    u.w = bfly(u.w, lm, hi);
  }
  if (hsz >= 16) {
    const float s = __fdiv_rn(1.0f, __fsqrt_rn((float)hsz));
    u = make_float4(__fmul_rn(u.x, s), __fmul_rn(u.y, s), __fmul_rn(u.z, s), __fmul_rn(u.w, s));
  }
  return u;
}

// Row r of a prep item by one warp: rotate, per-row int8 quantisation
// (fgm_quant_act, ops.c:181-204), the packed-tile row (ops.c:302-313).
// Rows past M write the zero padding of the last tile block.
__device__ void prep_row(const WlItem &it, int r, int M, int lane) {
  const int K = it.K, KB = K >> 6, nch = K >> 7;
  int8_t *pa_row = it.pa + ((size_t)(r >> 4) * KB) * kATile + (size_t)(r & 15) * 64;
  if (r >= M) {
    for (int c = 0; c < nch; c++) {
      const int kk = c * 128 + lane * 4;
      *reinterpret_cast<uint32_t *>(pa_row + (size_t)(kk >> 6) * kATile + (kk & 63)) = 0u;
    }
    return;
  }
  const float *src = it.src + (size_t)r * it.lda + lane * 4;
  constexpr int kB = 8;  // chunks loaded together
  float mx = 0.0f;
  for (int c0 = 0; c0 < nch; c0 += kB) {
    float4 v[kB];
#pragma unroll
    for (int u = 0; u < kB; u++)
      if (c0 + u < nch) v[u] = *reinterpret_cast<const float4 *>(src + (c0 + u) * 128);
#pragma unroll
    for (int u = 0; u < kB; u++) {
      if (c0 + u >= nch) continue;
      const float4 x = fwht128(v[u], it.hsz, lane);
      const float a0 = fabsf(x.x), a1 = fabsf(x.y), a2 = fabsf(x.z), a3 = fabsf(x.w);
      mx = a0 > mx ? a0 : mx;
      mx = a1 > mx ? a1 : mx;
      mx = a2 > mx ? a2 : mx;
      mx = a3 > mx ? a3 : mx;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float u = __shfl_xor_sync(0xffffffffu, mx, o);
    mx = u > mx ? u : mx;
  }
  const float s = (mx == 0.0f) ? 1.0f : __fdiv_rn(mx, 127.0f);
  const float inv = __fdiv_rn(1.0f, s);
  for (int c0 = 0; c0 < nch; c0 += kB) {
    float4 v[kB];
#pragma unroll
    for (int u = 0; u < kB; u++)
      if (c0 + u < nch) v[u] = *reinterpret_cast<const float4 *>(src + (c0 + u) * 128);
#pragma unroll
    for (int u = 0; u < kB; u++) {
      if (c0 + u >= nch) continue;
      const int kk = (c0 + u) * 128 + lane * 4;
      *reinterpret_cast<uint32_t *>(pa_row + (size_t)(kk >> 6) * kATile + (kk & 63)) =
          q8_quad(fwht128(v[u], it.hsz, lane), inv);
    }
  }
  if (lane == 0) it.qs[r] = s;
}

// ------------------------------------------------------- cooperative rows
// The preps that depend on nothing in the list (their inputs were written
// before the run) are prepared at the start of the run by every CTA's
// consumer warps together: the host deals their real rows (rows past M are
// never read by the list's GEMMs) to the CTAs by cost, each CTA a few rows.
// The consumer warps first fill their weight rings (the weights never come
// from earlier kernels, so they stream while a previous launch finishes),
// then walk the (row, 128-value chunk) pairs of the CTA's rows with a
// stride of one warp each: a first pass keeps each row's largest |x| in
// shared memory, a second pass quantises.  The CTA then publishes its rows.
constexpr int kCoopRows = kWlCoopRows;
constexpr int kCoopBatch = 8;  // chunks a warp loads together (its first batch stays held)
using CoopRow = WlCoopRow;

__device__ __forceinline__ void consumers_sync(int W) {
  asm volatile("bar.sync 1, %0;" ::"r"(W * 32) : "memory");
}

// The CTA's row descriptors into shared memory (one warp, lane k: row k;
// one load each), the rows' chunk offsets and cleared maxima.
__device__ __forceinline__ void coop_fetch(const WlParams &p, int nr, int lane, CoopRow *rows,
                                           int *cstart, unsigned *rmax) {
  int nch = 0;
  if (lane < nr) {
    const CoopRow cr = p.coop[(size_t)blockIdx.x * kCoopRows + lane];
    rows[lane] = cr;
    rmax[lane] = 0u;
    nch = cr.nch;
  }
  // exclusive prefix of the chunk counts
  int incl = nch;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane < nr) cstart[lane + 1] = incl;
  if (lane == 0) cstart[0] = 0;
}

__device__ __forceinline__ int coop_row_of(const int *cstart, int nr, int id) {
  int k = 0;
  while (k + 1 < nr && cstart[k + 1] <= id) k++;
  return k;
}

// Load the warp's batch starting at chunk id b0 (stride W) of the CTA's rows.
__device__ __forceinline__ void coop_load(const CoopRow *rows, const int *cstart, int nr, int T,
                                          int b0, int W, int lane, float4 (&v)[kCoopBatch],
                                          int (&kk)[kCoopBatch], int (&cc)[kCoopBatch]) {
#pragma unroll
  for (int u = 0; u < kCoopBatch; u++) {
    const int id = b0 + u * W;
    kk[u] = -1;
    if (id < T) {
      const int k = coop_row_of(cstart, nr, id);
      cc[u] = id - cstart[k];
      v[u] = *reinterpret_cast<const float4 *>(rows[k].src + cc[u] * 128 + lane * 4);
      kk[u] = k;
    }
  }
}

__device__ __forceinline__ void coop_max(const CoopRow *rows, unsigned *rmax, int lane,
                                         const float4 (&v)[kCoopBatch],
                                         const int (&kk)[kCoopBatch]) {
#pragma unroll
  for (int u = 0; u < kCoopBatch; u++) {
    if (kk[u] < 0) continue;  // warp-uniform
    const float4 x = fwht128(v[u], rows[kk[u]].hsz, lane);
    float m = fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    // |x| >= 0 orders as its bits; a NaN maximum (every lane NaN) is
    // skipped, as the per-row prep's comparisons skip NaNs
    if (lane == 0 && m == m) atomicMax(&rmax[kk[u]], __float_as_uint(m));
  }
}

__device__ __forceinline__ void coop_quant(const CoopRow *rows, const unsigned *rmax, int lane,
                                           const float4 (&v)[kCoopBatch],
                                           const int (&kk)[kCoopBatch],
                                           const int (&cc)[kCoopBatch]) {
#pragma unroll
  for (int u = 0; u < kCoopBatch; u++) {
    if (kk[u] < 0) continue;
    const CoopRow &cr = rows[kk[u]];
    const float m = __uint_as_float(rmax[kk[u]]);
    const float sc = (m == 0.0f) ? 1.0f : __fdiv_rn(m, 127.0f);
    const int kq = cc[u] * 128 + lane * 4;
    *reinterpret_cast<uint32_t *>(cr.pa_row + (size_t)(kq >> 6) * kATile + (kq & 63)) =
        q8_quad(fwht128(v[u], cr.hsz, lane), __fdiv_rn(1.0f, sc));
  }
}

// The CTA's rows, by every consumer warp (cw of W), in two calls: coop_first
// issues the warp's first batch of chunks (held in registers until the end);
// coop_rows, called once the weight rings are out, walks the rest, meets the
// row maxima, quantises and publishes.  A CTA with at most kCoopBatch chunks
// per warp reads its rows once.
__device__ __forceinline__ void coop_first(int cw, int W, int lane, int nr, const CoopRow *rows,
                                           const int *cstart, float4 (&h)[kCoopBatch],
                                           int (&hk)[kCoopBatch], int (&hc)[kCoopBatch]) {
  coop_load(rows, cstart, nr, cstart[nr], cw, W, lane, h, hk, hc);
}

__device__ void coop_rows(const WlParams &p, int cw, int W, int lane, int nr, const CoopRow *rows,
                          const int *cstart, unsigned *rmax, const float4 (&h)[kCoopBatch],
                          const int (&hk)[kCoopBatch], const int (&hc)[kCoopBatch]) {
  const int T = cstart[nr];
  // pass 1: each row's largest |x| after the rotation
  for (int b0 = cw + kCoopBatch * W; b0 < T; b0 += kCoopBatch * W) {
    float4 v[kCoopBatch];
    int kk[kCoopBatch], cc[kCoopBatch];
    coop_load(rows, cstart, nr, T, b0, W, lane, v, kk, cc);
    coop_max(rows, rmax, lane, v, kk);
  }
  coop_max(rows, rmax, lane, h, hk);
  consumers_sync(W);
  // pass 2: quantise (the held batch from registers, later ones from L2)
  coop_quant(rows, rmax, lane, h, hk, hc);
  for (int b0 = cw + kCoopBatch * W; b0 < T; b0 += kCoopBatch * W) {
    float4 v[kCoopBatch];
    int kk[kCoopBatch], cc[kCoopBatch];
    coop_load(rows, cstart, nr, T, b0, W, lane, v, kk, cc);
    coop_quant(rows, rmax, lane, v, kk, cc);
  }
  if (cw == 0 && lane < nr) {
    const float m = __uint_as_float(rmax[lane]);
    *rows[lane].qs = (m == 0.0f) ? 1.0f : __fdiv_rn(m, 127.0f);
  }
  // publish: the packed rows are read by TMA loads (async proxy) in other CTAs
  fence_proxy_async_global();
  __threadfence();
  consumers_sync(W);
  if (cw == 0 && lane < nr) atomicAdd(p.done + rows[lane].item, rows[lane].pub);
}

// ------------------------------------------------------------ unit queue
// The consumer warps of a CTA take the units of its segments, in list order,
// from one shared counter at the moment their weight rings need them (a warp
// that runs ahead takes more), and remember them in a small queue of their
// own for the compute side.  Taking units in list order keeps the segments in
// order: a warp finishes its units of segment g before any later unit.
constexpr int kWlFifo = 16;  // units a warp may hold ahead of its compute (> stages + 1)

struct Issue {            // the issue side of a consumer warp
  int j, total;           // next CTA-local unit index taken; the CTA's units
  int si, seg_end;        // segment of unit j, and the CTA-local index past it
  int st, nst;            // stage of the current unit, stages per unit
  int nb;                 // current n-block
  const uint8_t *B;       // weights of the current segment's item
  const CUtensorMap *smap;  // its int4 scale view
  int ubytes, rows_st, nb0, kind;
  bool live;              // a unit with weight stages is current
  bool loaded;            // the fields above belong to segment si
};

// Segment index and item fields for CTA-local unit j (segments advance monotonically).
__device__ __forceinline__ void issue_seg(Issue &q, const WlParams &p, const WlSeg *segs,
                                          int nseg, int &seg_lo) {
  if (q.j < q.seg_end && q.loaded) return;  // same segment: the cached fields hold
  while (q.si < nseg && q.j >= q.seg_end) {
    seg_lo = q.seg_end;
    q.si++;
    if (q.si < nseg) q.seg_end += segs[q.si].nu;
  }
  if (q.si >= nseg) return;
  const WlSeg &sg = segs[q.si];
  q.nst = sg.nst;
  q.B = sg.B;
  q.smap = sg.smap;
  q.ubytes = sg.ubytes;
  q.rows_st = sg.rows_st;
  q.nb0 = sg.nb_base;  // n-block of the segment's first unit
  q.kind = sg.kind;
  q.loaded = true;
}

template <int MT>
__global__ void __launch_bounds__((kWlMaxWarps + 1) * 32, 1) worklist_kernel(const WlParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ uint64_t s_full[kWlASlots], s_empty[kWlASlots];
  __shared__ uint64_t s_ring[kWlMaxWarps][kWlMaxStages];
  __shared__ float s_as[kWlASlots][16];
  __shared__ uint32_t s_aoff[kWlASlots];
  __shared__ int s_r0[kWlASlots], s_r1[kWlASlots];  // producer: regions of the last four segments
  __shared__ int s_grab;                            // next CTA-local unit to hand out
  __shared__ int s_left[kWlASlots];                 // units of a GEMM segment still unfinished
  __shared__ int s_fifo[kWlMaxWarps][kWlFifo];      // each warp's taken units, in order
  __shared__ CoopRow s_crow[kCoopRows];              // cooperative rows: their descriptors,
  __shared__ int s_cstart[kCoopRows + 1];            // first chunk of each,
  __shared__ unsigned s_rmax[kCoopRows];             // largest |x| of each (as bits)
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const WlSeg *segs = p.segs + p.seg_off[blockIdx.x];
  const int nseg = p.seg_off[blockIdx.x + 1] - p.seg_off[blockIdx.x];
  const int S = p.stages, W = p.warps;
  const uint32_t abuf0 = tc::smem_u32(smem);
  const uint32_t ring0 = abuf0 + (uint32_t)p.a_ring;

  // barriers: one thread each (the ring's W x S, then the slots' full and empty)
  if ((int)threadIdx.x < W * S) {
    tc::mbar_init(&s_ring[threadIdx.x / S][threadIdx.x % S], 1);
    tc::fence_mbar_init();
  } else if ((int)threadIdx.x < W * S + kWlASlots) {
    const int b = threadIdx.x - W * S;
    tc::mbar_init(&s_full[b], 1);
    tc::mbar_init(&s_empty[b], 1);  // the warp finishing a segment's last unit arrives
    tc::fence_mbar_init();
  }
  if (threadIdx.x == 0) s_grab = 0;
  __syncthreads();
  pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // GEMM segment g stages its activations in slot g % 4 (barriers, scales)
    // at a region of the activation ring; a region is reused once every unit
    // of the segments holding it is done.
    // The entries' descriptors and the segments' activation maps are list
    // data: prefetched while the previous kernel finishes.
    for (size_t o = (size_t)lane * 128; o < (size_t)p.n_items * sizeof(WlItem); o += 32 * 128)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<const char *>(p.items) + o));
    for (int si = lane; si < nseg; si += 32)
      if (segs[si].kind != kWlPrep) tc::prefetch_tmap(&p.items[segs[si].item].amap);
    pdl_wait();  // packed activations and their scales may come from earlier kernels
    int g = 0, head = 0;
    bool ok = true;
    for (int si = 0; si < nseg && ok; si++) {
      const WlSeg &sg = segs[si];
      if (sg.kind == kWlPrep) continue;
      const WlItem &it = p.items[sg.item];
      const int b = g & (kWlASlots - 1);
      const int bytes = it.K / 64 * MT * 512;
      const int sz = (bytes + 1023) & ~1023;
      if (g >= kWlASlots)  // segment g - 4, the slot's last user, is done
        ok = wl_wait(&s_empty[b], (uint32_t)(((g >> 2) - 1) & 1), p);
      // The region: the first of the head, the ring start or the end of a
      // live younger segment's region where the block fits without touching
      // a region still in use (a large block held by a long segment does not
      // hold up the small ones behind it).  Lane 0 decides.
      int off = -1;
      if (ok && lane == 0) {
        const uint64_t t0 = tc::globaltimer_ns();
        while (off < 0) {
          int cand[kWlASlots + 1];
          int nc = 0;
          cand[nc++] = head;
          cand[nc++] = 0;
          for (int j = g - kWlASlots + 1; j < g; j++)
            if (j >= 0) cand[nc++] = s_r1[j & (kWlASlots - 1)];
          for (int k = 0; k < nc && off < 0; k++) {
            const int x = cand[k];
            if (x + sz > p.a_ring) continue;
            bool fit = true;
            for (int j = g - kWlASlots + 1; j < g && fit; j++) {
              if (j < 0) continue;
              const int jb = j & (kWlASlots - 1);
              if (s_r0[jb] < x + sz && x < s_r1[jb] &&
                  !tc::mbar_try_wait(&s_empty[jb], (uint32_t)((j >> 2) & 1)))
                fit = false;
            }
            if (fit) off = x;
          }
          if (off < 0 && (ld_volatile(p.abort) || tc::globaltimer_ns() - t0 > kWlLimitNs)) break;
        }
        ok = off >= 0;
      }
      off = __shfl_sync(0xffffffffu, off, 0);
      if (ok && lane == 0) ok = wl_wait_item(p, it.deps[0]) && wl_wait_item(p, it.deps[1]);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
      __syncwarp();
      if (lane == 0) {
        s_r0[b] = off;
        s_r1[b] = off + sz;
        s_left[b] = sg.nu;  // the slot's previous segment is done; seen by its units
                            // through the full barrier this lane arms below
      }
      head = off + sz;
      fence_proxy_async_global();  // the activations may have been written in this launch
      if (lane < 16) s_as[b][lane] = lane < p.M ? it.a_scale[lane] : 0.0f;
      if (lane == 0) s_aoff[b] = (uint32_t)off;
      __syncwarp();
      if (lane == 0) {
        tc::mbar_expect_tx(&s_full[b], (uint32_t)bytes);
        tc::tma_load_3d(smem + off, &it.amap, &s_full[b], 0, 0, 0);
      }
      g++;
    }
    if (!ok) {
      if (lane == 0) wl_fail(p, 5);
      // the last activation boxes requested may still be landing
      for (int k = (g > kWlASlots ? g - kWlASlots : 0); k < g; k++)
        tc::mbar_wait(&s_full[k & (kWlASlots - 1)], (uint32_t)((k >> 2) & 1));
    }
  } else if (warp <= W) {
    // ------------------------------------------------------------ consumers
    const int cw = warp - 1;
    const WlLane L = make_lane(lane);
    const uint32_t ring = ring0 + (uint32_t)(cw * S * kWlStage);
    uint64_t *bars = s_ring[cw];
    int *fifo = s_fifo[cw];
    int total = 0;
    for (int si = 0; si < nseg; si++) total += segs[si].nu;
    Issue q{};
    q.total = total;
    q.si = 0;
    q.seg_end = nseg ? segs[0].nu : 0;
    int seg_lo = 0, fpush = 0, fpop = 0, islot = 0, inflight = 0;
    bool exhausted = false;  // every unit of the CTA has been taken
    // Take the next unit for this warp and push it on its queue (the caller
    // checked there is room); units without weight stages (prep rows) are
    // only queued.
    auto take = [&]() {
      int j = 0;
      if (lane == 0) j = atomicAdd(&s_grab, 1);
      j = __shfl_sync(0xffffffffu, j, 0);
      if (j >= total) {
        exhausted = true;
        q.live = false;
        return;
      }
      q.j = j;
      issue_seg(q, p, segs, nseg, seg_lo);
      if (lane == 0) fifo[fpush & (kWlFifo - 1)] = j;
      fpush++;
      q.st = 0;
      q.live = q.kind != kWlPrep;
      if (q.live) q.nb = q.nb0 + (j - seg_lo);
    };
    // Make a unit with weight stages current on the issue side, taking units
    // while the queue has room.
    auto refill = [&]() {
      while (!q.live && !exhausted && fpush - fpop < kWlFifo - 1) take();
    };
    auto next_live = [&]() {
      q.live = false;
      refill();
    };
    // The stage at the issue side into ring slot islot: its weight tiles (one
    // bulk copy) and, for int4, the f16 scale rows of its groups (one 2-D
    // TMA box of 16 columns x the stage's groups) behind them.
    auto issue = [&]() {
      const uint32_t dst = ring + islot * kWlStage;
      if (lane == 0) {
        const int rows = q.rows_st;
        tc::mbar_expect_tx(&bars[islot], (uint32_t)(kWlStageW + rows * 32));
        bulk_g2s(dst, q.B + (size_t)q.nb * q.ubytes + (size_t)q.st * kWlStageW, kWlStageW,
                 &bars[islot]);
        if (rows)
          tma_load_2d_u32(dst + kWlStageW, q.smap, &bars[islot], q.nb * 16, q.st * rows);
      }
      if (++islot == S) islot = 0;
      inflight++;
      if (++q.st == q.nst) next_live();
    };
    auto can_issue = [&]() { return q.live; };

    // the weights never come from earlier kernels: fill the ring first, then
    // this CTA's share of the dependency-free preps' rows (their descriptors
    // are list data, fetched before waiting for the previous kernel)
    // This CTA's share of the dependency-free preps' rows: their descriptors
    // (list data), then -- once earlier kernels are done -- the rows' loads,
    // ahead of the weight rings in the memory queues; the weights then
    // stream while the rows are quantised.
    const int cnr = p.coop_n[blockIdx.x];
    if (cw == 0 && cnr > 0) coop_fetch(p, cnr, lane, s_crow, s_cstart, s_rmax);
    pdl_wait();  // prep sources and GEMM outputs are ordered after earlier kernels
    float4 ch[kCoopBatch];
    int chk[kCoopBatch], chc[kCoopBatch];
    if (cnr > 0) {
      consumers_sync(W);  // the descriptors
      coop_first(cw, W, lane, cnr, s_crow, s_cstart, ch, chk, chc);
    }
    refill();
    while (inflight < S && can_issue()) issue();
    if (cnr > 0) coop_rows(p, cw, W, lane, cnr, s_crow, s_cstart, s_rmax, ch, chk, chc);

    bool ok = true;
    int cseg = 0, cseg_lo = 0, cseg_end = nseg ? segs[0].nu : 0;  // compute side's segment
    int cslot = 0;
    uint32_t cpar = 0;
    while (ok) {
      if (fpop == fpush) {  // nothing taken: take more
        if (exhausted) break;
        refill();
        while (inflight < S && can_issue()) issue();
        continue;
      }
      const int j = fifo[fpop & (kWlFifo - 1)];
      fpop++;
      refill();  // there is room again
      while (j >= cseg_end) {
        cseg_lo = cseg_end;
        cseg++;
        cseg_end += segs[cseg].nu;
      }
      const WlSeg &sg = segs[cseg];
      const int kind = sg.kind;
      if (kind == kWlPrep) {
        const WlItem &it = p.items[sg.item];
        if (lane == 0) ok = wl_wait_item(p, it.deps[0]) && wl_wait_item(p, it.deps[1]);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
        prep_row(it, sg.ub + (j - cseg_lo), p.M, lane);
        if (it.waited) wl_signal(p, sg.item, 1u, lane);
        continue;
      }
      const int gseq = sg.gseq, nst = sg.nst, ldc = sg.ldc, c0 = sg.c_col0, gk = sg.gk;
      const int nb = sg.nb_base + (j - cseg_lo);
      float *C = sg.C;
      const float *b_scale8 = static_cast<const float *>(sg.b_scale);
      const int b = gseq & (kWlASlots - 1);
      ok = __all_sync(0xffffffffu, wl_wait(&s_full[b], (uint32_t)((gseq >> 2) & 1), p));
      if (!ok) break;
      const uint32_t ab = abuf0 + s_aoff[b];
      // one code path per weight format and int4 scale group
      auto run = [&](auto kind_tag) {
        constexpr int KIND = decltype(kind_tag)::value;
        constexpr bool Q4 = KIND != 0;
        constexpr uint32_t a_step = (Q4 ? 8 : 4) * MT * 512;  // activation bytes per stage
        float2 cf[MT][2];  // running int4 sums: values (i = 0, 1) and (i = 2, 3)
        int32_t acc[MT][4];
#pragma unroll
        for (int mt = 0; mt < MT; mt++) {
          cf[mt][0] = cf[mt][1] = make_float2(0.0f, 0.0f);
#pragma unroll
          for (int i = 0; i < 4; i++) acc[mt][i] = 0;
        }
        float bs0 = 0.0f, bs1 = 0.0f;  // int8 per-channel scales of columns g8, g8 + 8
        if (!Q4) {
          bs0 = __ldg(b_scale8 + nb * 16 + L.g8);
          bs1 = __ldg(b_scale8 + nb * 16 + L.g8 + 8);
        }
        uint32_t abs_ = ab;
        for (int st = 0; st < nst; st++) {
          ok = __all_sync(0xffffffffu, wl_wait(&bars[cslot], cpar, p));
          if (!ok) return;
          const uint32_t stg = ring + cslot * kWlStage;
          if constexpr (Q4) q4_stage<MT, (Q4 ? KIND : 1)>(stg, abs_, L, cf);
          else q8_stage<MT>(stg, abs_, L, acc);
          abs_ += a_step;
          __syncwarp();
          fence_proxy_async_smem();  // this warp's reads of the slot precede its refill
          inflight--;
          if (++cslot == S) {
            cslot = 0;
            cpar ^= 1u;
          }
          if (can_issue()) issue();
        }
#pragma unroll
        for (int mt = 0; mt < MT; mt++)
#pragma unroll
          for (int i = 0; i < 4; i++) {
            const int m = mt * 8 + 2 * L.tig + (i & 1);
            const int n = nb * 16 + L.g8 + (i >= 2 ? 8 : 0);
            if (m >= p.M) continue;
            const float as = s_as[b][m];
            const float2 c2 = cf[mt][i >> 1];
            C[(size_t)m * ldc + (n - c0)] =
                Q4 ? __fmul_rn((i & 1) ? c2.y : c2.x, as)
                   : __fmul_rn(__int2float_rn(acc[mt][i]), __fmul_rn(i < 2 ? bs0 : bs1, as));
          }
      };
      if (kind == kWlQ8) run(std::integral_constant<int, 0>{});
      else if (gk == 1) run(std::integral_constant<int, 1>{});
      else if (gk == 2) run(std::integral_constant<int, 2>{});
      else if (gk == 4) run(std::integral_constant<int, 4>{});
      else run(std::integral_constant<int, 8>{});
      if (!ok) break;
      // This unit is done.  The warp that finishes the segment's last unit
      // releases its activation region; if another item waits for this one,
      // every unit's outputs are made visible first and the segment is
      // published.
      const bool waited = sg.waited != 0;
      __syncwarp();
      if (lane == 0) {
        if (waited) __threadfence();
        if (atomicAdd(&s_left[b], -1) == 1) {
          if (waited) {
            __threadfence();
            atomicAdd(p.done + segs[cseg].item, (unsigned)segs[cseg].nu);
          }
          asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::smem_u32(&s_empty[b]))
                       : "memory");
        }
      }
      // keep the ring full when the queue was the limit
      while (inflight < S && can_issue()) issue();
    }
    if (!ok) {
      if (lane == 0) wl_fail(p, 5);
      // weight stages still in flight land before the CTA exits
      for (int k = 0; k < inflight; k++) {
        tc::mbar_wait(&bars[cslot], cpar);
        if (++cslot == S) {
          cslot = 0;
          cpar ^= 1u;
        }
      }
    }
  }

  // ---- the last CTA to finish resets the counters for the next launch
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(p.ctas_done, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence();
      for (int i = 0; i < p.n_items; i++) p.done[i] = 0;
      *p.abort = 0;
      *p.ctas_done = 0;
      __threadfence();
    }
  }
}

}  // namespace

// ======================================================================= host
static size_t worklist_smem(int a_ring, int warps, int stages) {
  return 1024 + (size_t)a_ring + (size_t)warps * stages * kWlStage;
}

static int wl_static_smem(int MT) {
  cudaFuncAttributes a{};
  const cudaError_t e = MT == 1 ? cudaFuncGetAttributes(&a, worklist_kernel<1>)
                                : cudaFuncGetAttributes(&a, worklist_kernel<2>);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return 4096;
  }
  return (int)a.sharedSizeBytes;
}

const char *worklist_plan(WlPlan &pl, std::vector<WlItem> &items, int M, int num_sms,
                          size_t smem_optin) {
  const int n = (int)items.size();
  pl.M = M;
  pl.MT = M <= 8 ? 1 : 2;
  pl.grid = num_sms;
  // ---- shared memory: the activation ring and the consumers' weight rings.
  // The most consumer warps (latency hiding) whose two-stage rings leave the
  // activation ring room for the widest segment and two of the narrowest (a
  // CTA holding a wide block keeps staging the blocks behind it), else for
  // the widest alone; FGM_CUDA_WORKLIST_WARPS (8..15) caps the count.
  int max_seg = 1024, min_seg = 1 << 30;
  for (const WlItem &it : items)
    if (it.kind != kWlPrep) {
      const int sz = (it.K / 64 * pl.MT * 512 + 1023) & ~1023;
      max_seg = std::max(max_seg, sz);
      min_seg = std::min(min_seg, sz);
    }
  if (min_seg > max_seg) min_seg = max_seg;
  const size_t limit = smem_optin + 1024 - (size_t)wl_static_smem(pl.MT) - 256;
  int want = 0;
  if (const char *e = getenv("FGM_CUDA_WORKLIST_WARPS")) want = atoi(e);
  pl.warps = 0;
  for (int pass = 0; pass < 2 && !pl.warps; pass++)
  for (int w = kWlMaxWarps; w >= 8; w--) {
    if (want && w > want) continue;
    const size_t rings = (size_t)w * 2 * kWlStage;
    const size_t need = (size_t)max_seg + (pass == 0 && max_seg > min_seg ? 2 * (size_t)min_seg : 0);
    if (1024 + rings + need > limit) continue;
    pl.warps = w;
    pl.stages = 2;
    // deeper rings while the activation ring still holds two widest segments
    while (pl.stages < kWlMaxStages &&
           1024 + (size_t)w * (pl.stages + 1) * kWlStage + 2 * (size_t)max_seg <= limit)
      pl.stages++;
    pl.a_ring = (int)((limit - 1024 - (size_t)w * pl.stages * kWlStage) & ~(size_t)1023);
    break;
  }
  if (!pl.warps) return "the activations of the widest item do not fit in shared memory";
  pl.smem = worklist_smem(pl.a_ring, pl.warps, pl.stages);

  // ---- preps that depend on nothing: their real rows go to the CTAs,
  // longest rows first to the least loaded CTA (at most kCoopRows each);
  // every CTA's consumer warps prepare its rows at the start of the run and
  // the entries that read them wait for their counters.  Rows past M are
  // not written (the list's GEMMs read rows [0, M) only).
  std::vector<char> pro(n, 0);
  {
    std::vector<std::pair<int, int>> jobs;  // (K, item*16 + row)
    for (int i = 0; i < n; i++) {
      const WlItem &it = items[i];
      if (it.kind != kWlPrep || it.deps[0] >= 0 || it.deps[1] >= 0) continue;
      if ((long)jobs.size() + M > (long)kCoopRows * num_sms) break;  // the rest run as units
      pro[i] = 1;
      for (int r = 0; r < M; r++) jobs.push_back({it.K, i * 16 + r});
    }
    std::stable_sort(jobs.begin(), jobs.end(),
                     [](const std::pair<int, int> &a, const std::pair<int, int> &b) {
                       return a.first > b.first;
                     });
    std::vector<long> load(num_sms, 0);
    std::vector<std::vector<int>> rows(num_sms);
    for (const auto &j : jobs) {
      int best = -1;
      for (int c = 0; c < num_sms; c++)
        if ((int)rows[c].size() < kCoopRows && (best < 0 || load[c] < load[best])) best = c;
      rows[best].push_back(j.second);
      load[best] += j.first;
    }
    pl.coop.assign((size_t)num_sms * kCoopRows, WlCoopRow{});
    pl.coop_n.assign(num_sms, 0);
    for (int c = 0; c < num_sms; c++) {
      pl.coop_n[c] = (int)rows[c].size();
      for (int k = 0; k < (int)rows[c].size(); k++) {
        const int job = rows[c][k], r = job & 15;
        const WlItem &it = items[job >> 4];
        WlCoopRow &cr = pl.coop[(size_t)c * kCoopRows + k];
        cr.src = it.src + (size_t)r * it.lda;
        cr.pa_row = it.pa + (size_t)r * 64;  // one 16-row tile block (M <= 16)
        cr.qs = it.qs + r;
        cr.item = job >> 4;
        cr.hsz = it.hsz;
        cr.pub = 1u + (r == 0 ? (unsigned)(it.units - M) : 0u);
        cr.nch = it.K >> 7;
      }
    }
  }
  for (WlItem &it : items) it.waited = 0;
  for (const WlItem &it : items)
    for (int d : it.deps)
      if (d >= 0) items[d].waited = 1;
  // ---- levels: one more than the deepest dependency
  std::vector<int> level(n, 0);
  int nlev = 0;
  for (int i = 0; i < n; i++) {
    for (int d : items[i].deps)
      if (d >= 0) level[i] = std::max(level[i], level[d] + 1);
    nlev = std::max(nlev, level[i] + 1);
  }
  // Cost of one unit in 4 KB weight stages: its stages plus a fixed cost per
  // unit (taking it, its epilogue) measured at about one and a half stages;
  // a prep row: two passes over its f32 source, which one warp reads at a
  // fraction of the weight rate.
  auto unit_cost = [&](const WlItem &it, int u) -> double {
    if (it.kind == kWlQ4) return it.K / 512 + 1.5;
    if (it.kind == kWlQ8) return it.K / 256 + 1.5;
    return u < M ? 3.0 * it.K / 1024 : 1.0;
  };
  // ---- each CTA's (item, unit range) pieces, level by level
  const int G = num_sms;
  struct Piece {
    int item, u0, u1;
  };
  std::vector<std::vector<Piece>> cta(G);
  int rr = 0;  // round-robin position of prep rows
  for (int lv = 0; lv < nlev; lv++) {
    std::vector<size_t> first(G);  // where this level's pieces start in each CTA's list
    for (int c = 0; c < G; c++) first[c] = cta[c].size();
    for (int i = 0; i < n; i++) {  // prep rows round-robin over the CTAs
      if (level[i] != lv || pro[i] || items[i].kind != kWlPrep) continue;
      for (int u = 0; u < items[i].units; u++, rr++) cta[rr % G].push_back(Piece{i, u, u + 1});
    }
    // GEMM units.  Items whose units cost more than twice the level's
    // cheapest units ("large": e.g. the K=8192 down projections) each get a
    // set of CTAs of their own, filling about half of each CTA's share, so
    // no CTA holds two large activation blocks or ends on large units alone;
    // the other items' units then fill every CTA's remaining share in
    // contiguous ranges, in list order.  (Inside each CTA the large units go
    // first, see below.)
    double total = 0, cheapest = 1e30;
    for (int i = 0; i < n; i++)
      if (level[i] == lv && !pro[i] && items[i].kind != kWlPrep) {
        total += items[i].units * unit_cost(items[i], 0);
        cheapest = std::min(cheapest, unit_cost(items[i], 0));
      }
    const double share = total / G;
    std::vector<double> have(G, 0.0);
    std::vector<char> placed(n, 0);
    int next = 0;  // first CTA without a large item
    for (int i = 0; i < n; i++) {
      const WlItem &it = items[i];
      if (level[i] != lv || pro[i] || it.kind == kWlPrep) continue;
      const double cost = unit_cost(it, 0);
      if (cost <= 2 * cheapest) continue;
      int k = (int)std::lround(it.units * cost / (0.5 * share));
      k = std::max(1, std::min(k, it.units));
      if (next + k > G) break;  // out of CTAs: the rest are dealt like the others
      for (int j = 0; j < k; j++) {
        const int u0 = (int)((long)it.units * j / k), u1 = (int)((long)it.units * (j + 1) / k);
        if (u1 > u0) cta[next + j].push_back(Piece{i, u0, u1});
        have[next + j] += (u1 - u0) * cost;
      }
      next += k;
      placed[i] = 1;
    }
    std::vector<double> room_end(G + 1, 0.0);  // prefix of the CTAs' remaining shares
    for (int c = 0; c < G; c++) room_end[c + 1] = room_end[c] + std::max(0.0, share - have[c]);
    double rest = 0;  // the other items' cost, spread over the remaining shares
    for (int i = 0; i < n; i++)
      if (level[i] == lv && !pro[i] && items[i].kind != kWlPrep && !placed[i])
        rest += items[i].units * unit_cost(items[i], 0);
    if (room_end[G] <= 0)  // no room left anywhere: spread evenly
      for (int c = 0; c < G; c++) room_end[c + 1] = room_end[c] + 1.0;
    const double scale = rest > 0 ? room_end[G] / rest : 1.0;
    // the largest items first: the CTAs holding a large item's block (they
    // come first) then fill their room from one range of a big item, and
    // the many small items go where the activation ring has room for them
    std::vector<int> order;
    for (int i = 0; i < n; i++)
      if (level[i] == lv && !pro[i] && items[i].kind != kWlPrep && !placed[i]) order.push_back(i);
    std::stable_sort(order.begin(), order.end(), [&](int x, int y) {
      return items[x].units * unit_cost(items[x], 0) > items[y].units * unit_cost(items[y], 0);
    });
    double acc = 0;
    for (int i : order) {
      const WlItem &it = items[i];
      const double cost = unit_cost(it, 0);
      int u = 0;
      while (u < it.units) {
        // the CTA whose remaining share holds the middle of this unit
        const double mid = (acc + 0.5 * cost) * scale;
        int c = (int)(std::upper_bound(room_end.begin() + 1, room_end.end(), mid) -
                      (room_end.begin() + 1));
        c = std::min(c, G - 1);
        int u1 = u + 1;
        while (u1 < it.units && (acc + (u1 - u + 0.5) * cost) * scale < room_end[c + 1]) u1++;
        cta[c].push_back(Piece{i, u, u1});
        acc += (u1 - u) * cost;
        u = u1;
      }
    }
    // Inside a level the items are independent: each CTA takes its prep rows
    // first, then its GEMM units from the largest to the smallest, so the
    // end of the level is made of small units that every warp can share
    // (a few large units at the end would run on a few warps alone).
    for (int c = 0; c < G; c++)
      std::stable_sort(cta[c].begin() + first[c], cta[c].end(), [&](const Piece &x, const Piece &y) {
        const double cx = items[x.item].kind == kWlPrep ? 1e30 : unit_cost(items[x.item], 0);
        const double cy = items[y.item].kind == kWlPrep ? 1e30 : unit_cost(items[y.item], 0);
        return cx > cy;
      });
  }
  // ---- each CTA's segments in order; its consumer warps take the units
  // from a shared counter while running
  pl.seg_off.assign(G + 1, 0);
  pl.segs.clear();
  for (int c = 0; c < G; c++) {
    pl.seg_off[c] = (int)pl.segs.size();
    int gseq = 0;
    for (const Piece &pc : cta[c]) {
      const WlItem &it = items[pc.item];
      WlSeg sg{};
      sg.item = pc.item;
      sg.kind = it.kind;
      sg.nst = it.kind == kWlQ4 ? it.K / 512 : (it.kind == kWlQ8 ? it.K / 256 : 0);
      sg.ub = pc.u0;
      sg.nu = pc.u1 - pc.u0;
      sg.gseq = it.kind == kWlPrep ? -1 : gseq++;
      if (it.kind != kWlPrep) {
        sg.nb_base = it.nb0 + pc.u0;
        sg.ldc = it.ldc;
        sg.c_col0 = it.c_col0;
        sg.gk = it.gk;
        sg.waited = it.waited;
        sg.ubytes = it.K * (it.kind == kWlQ4 ? 8 : 16);  // K/64 tiles of 512 or 1024 bytes
        sg.rows_st = it.kind == kWlQ4 ? 8 / it.gk : 0;
        sg.C = it.C;
        sg.b_scale = it.b_scale;
        sg.B = it.B;
        sg.smap = nullptr;  // set once the descriptors' device address is known
      }
      pl.segs.push_back(sg);
    }
  }
  pl.seg_off[G] = (int)pl.segs.size();
  return nullptr;
}

cudaError_t launch_worklist(const WlParams &p, const WlPlan &pl, bool pdl, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.grid);
  cfg.blockDim = dim3((pl.warps + 1) * 32);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (pl.MT == 1) {
    cudaError_t e = cudaFuncSetAttribute(worklist_kernel<1>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem);
    if (e != cudaSuccess) return e;
    return cudaLaunchKernelEx(&cfg, worklist_kernel<1>, p);
  }
  cudaError_t e = cudaFuncSetAttribute(worklist_kernel<2>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem);
  if (e != cudaSuccess) return e;
  return cudaLaunchKernelEx(&cfg, worklist_kernel<2>, p);
}

}  // namespace fgm
