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
// prep -- are spread over all CTAs: GEMM units as contiguous ranges of equal
// weight bytes (independent items of a level run side by side on different
// SMs), prep rows round-robin.  A CTA's share is a list of segments (item,
// unit range); inside a CTA the units of its segments go round-robin to the
// consumer warps.  Every warp walks its units in list order, so the lowest
// unfinished item can always progress: the kernel cannot deadlock while all
// CTAs are resident (grid = one CTA per SM).
//
// CTA roles
// ---------
// Warp 0 (producer) stages each GEMM segment's activations: it waits for the
// item's dependencies (counters in global memory, acquire loads), then one
// 3-D TMA box brings the segment's packed rows [tiles][rows][64 B] into one
// of two shared buffers with the 64-byte swizzle, so the consumers' B-fragment
// loads (k-quads t, 4+t, 8+t, 12+t of row g) hit 32 distinct banks.  Warps
// 1..8 (consumers) each own a ring of 4 KB stages (8 int4 or 4 int8 tiles),
// filled by cp.async.bulk and refilled as soon as a stage is consumed, across
// unit and item boundaries; the weight issue runs ahead of everything else,
// before griddepcontrol.wait.  The arithmetic per stage is the decode
// kernel's (gemv.cu): mma.sync m16n8k32 s8 with the weights as the A operand
// read straight from the tile layout, int32 group sums, and the fold
// C = fmaf((float)acc_g, s_g, C) over ascending groups, then * a_scale
// (amx_gemm.c:103-113, :365-371); int8: (float)acc * (b_scale * a_scale)
// (amx_gemm.c:399).  Bit-identical to the per-call kernels.
//
// Waits and failures
// ------------------
// Every wait (mbarriers, dependency counters) gives up after 2 s or as soon
// as another warp has raised the list's abort word; the kernel then raises
// the device error word, waits (bounded) for its own copies in flight and
// returns.  The last CTA to finish resets the counters for the next launch.

#include <cuda.h>

#include <algorithm>
#include <cstring>
#include <vector>

#include "fgm_common.cuh"
#include "fgm_internal.h"
#include "stream_ptx.cuh"
#include "tc_ptx.cuh"

namespace fgm {

namespace {

using namespace stream;

constexpr int kWlWarps = 8;        // consumer warps per CTA
constexpr int kWlStage = 4096;     // bytes per ring stage
constexpr int kWlMaxStages = 8;
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
__device__ __forceinline__ bool wl_wait(uint64_t *bar, uint32_t parity, const WlParams &p) {
  if (tc::mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = tc::globaltimer_ns();
  while (!tc::mbar_try_wait(bar, parity)) {
    if (ld_volatile(p.abort)) return false;
    if (tc::globaltimer_ns() - t0 > kWlLimitNs) return false;
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
__device__ __forceinline__ void q4_stage(uint32_t st, uint32_t ab, const WlLane &L, uint32_t sc0,
                                         uint32_t sc1, float (&cf)[MT][4]) {
  constexpr int CH = MT == 1 ? 8 : 4;  // tiles whose operands load together
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
      const int lg = t / GK;  // group inside the stage
      float s0, s1;
      scale_pair(lg < 4 ? sc0 : sc1, (lg & 3) * 8, L.g8, s0, s1);
#pragma unroll
      for (int mt = 0; mt < MT; mt++)
#pragma unroll
        for (int i = 0; i < 4; i++)
          cf[mt][i] = __fmaf_rn(i2f_exact(gacc[mt][i] >> 4), i < 2 ? s0 : s1, cf[mt][i]);
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

template <int MT>
__device__ __forceinline__ void q4_stage_gk(int gk, uint32_t st, uint32_t ab, const WlLane &L,
                                            uint32_t sc0, uint32_t sc1, float (&cf)[MT][4]) {
  switch (gk) {
    case 1: q4_stage<MT, 1>(st, ab, L, sc0, sc1, cf); break;
    case 2: q4_stage<MT, 2>(st, ab, L, sc0, sc1, cf); break;
    case 4: q4_stage<MT, 4>(st, ab, L, sc0, sc1, cf); break;
    default: q4_stage<MT, 8>(st, ab, L, sc0, sc1, cf); break;
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

// -------------------------------------------------------- unit cursor
// Position of a consumer warp in its own sequence of weight stages: segment
// si of the CTA's list, this warp's j-th unit of that segment, stage st.
struct Cur {
  int si, j, st;
};

__device__ __forceinline__ int first_of(const WlSeg &sg, int cw) {
  int f = (cw - sg.base) % kWlWarps;
  return f < 0 ? f + kWlWarps : f;
}

__device__ __forceinline__ int count_of(const WlSeg &sg, int cw) {
  const int n = sg.u1 - sg.u0 - first_of(sg, cw);
  return n > 0 ? (n + kWlWarps - 1) / kWlWarps : 0;
}

// Move to the next segment (from si on) that holds weight stages for this warp.
__device__ __forceinline__ void skip_to_gemm(Cur &c, const WlSeg *segs, int nseg, int cw) {
  while (c.si < nseg && (segs[c.si].kind == kWlPrep || count_of(segs[c.si], cw) == 0)) c.si++;
}

__device__ __forceinline__ void advance(Cur &c, const WlSeg *segs, int nseg, int cw) {
  const WlSeg &sg = segs[c.si];
  if (++c.st < sg.nst) return;
  c.st = 0;
  if (++c.j < count_of(sg, cw)) return;
  c.j = 0;
  c.si++;
  skip_to_gemm(c, segs, nseg, cw);
}

template <int MT>
__global__ void __launch_bounds__((kWlWarps + 1) * 32, 1) worklist_kernel(const WlParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ uint64_t s_full[2], s_empty[2];
  __shared__ uint64_t s_ring[kWlWarps][kWlMaxStages];
  __shared__ float s_as[2][16];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const WlSeg *segs = p.segs + p.seg_off[blockIdx.x];
  const int nseg = p.seg_off[blockIdx.x + 1] - p.seg_off[blockIdx.x];
  const int S = p.stages;
  const uint32_t abuf0 = tc::smem_u32(smem);
  const uint32_t ring0 = abuf0 + (uint32_t)(p.n_abuf * p.abuf_bytes);

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; b++) {
      tc::mbar_init(&s_full[b], 1);
      tc::mbar_init(&s_empty[b], kWlWarps);
    }
    for (int w = 0; w < kWlWarps; w++)
      for (int s = 0; s < S; s++) tc::mbar_init(&s_ring[w][s], 1);
    tc::fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    pdl_wait();  // packed activations and their scales may come from earlier kernels
    int g = 0, issued = 0;
    bool ok = true;
    for (int si = 0; si < nseg && ok; si++) {
      const WlSeg sg = segs[si];
      if (sg.kind == kWlPrep) continue;
      const WlItem &it = p.items[sg.item];
      const int b = g % p.n_abuf, r = g / p.n_abuf;
      if (r > 0) ok = wl_wait(&s_empty[b], (r - 1) & 1, p);  // every consumer left segment g - n_abuf
      if (ok && lane == 0) ok = wl_wait_item(p, it.deps[0]) && wl_wait_item(p, it.deps[1]);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
      fence_proxy_async_global();  // the activations may have been written in this launch
      if (lane < 16) s_as[b][lane] = lane < p.M ? it.a_scale[lane] : 0.0f;
      __syncwarp();
      if (lane == 0) {
        tc::mbar_expect_tx(&s_full[b], (uint32_t)(it.K / 64 * MT * 512));
        tc::tma_load_3d(smem + (size_t)b * p.abuf_bytes, &it.amap, &s_full[b], 0, 0, 0);
      }
      issued = ++g;
    }
    if (!ok) {
      if (lane == 0) wl_fail(p, 5);
      // the last activation boxes requested may still be landing
      for (int k = (issued > p.n_abuf ? issued - p.n_abuf : 0); k < issued; k++)
        tc::mbar_wait(&s_full[k % p.n_abuf], (k / p.n_abuf) & 1);
    }
  } else {
    // ------------------------------------------------------------ consumers
    const int cw = warp - 1;
    const WlLane L = make_lane(lane);
    const uint32_t ring = ring0 + (uint32_t)(cw * S * kWlStage);
    uint64_t *bars = s_ring[cw];
    Cur ic{0, 0, 0}, sc{0, 0, 0};
    skip_to_gemm(ic, segs, nseg, cw);
    skip_to_gemm(sc, segs, nseg, cw);
    int issued = 0, consumed = 0;
    auto issue = [&]() {  // next weight stage at the issue cursor into its ring slot
      const WlSeg &sg = segs[ic.si];
      const WlItem &it = p.items[sg.item];
      const int KB = it.K >> 6, T = it.kind == kWlQ4 ? 8 : 4, TB = it.kind == kWlQ4 ? 512 : 1024;
      const int nb = it.nb0 + sg.u0 + first_of(sg, cw) + ic.j * kWlWarps;
      const int slot = issued % S;
      if (lane == 0) {
        tc::mbar_expect_tx(&bars[slot], kWlStage);
        bulk_g2s(ring + slot * kWlStage, it.B + ((size_t)nb * KB + (size_t)ic.st * T) * TB,
                 kWlStage, &bars[slot]);
      }
      issued++;
      advance(ic, segs, nseg, cw);
    };
    // int4 scales of the stage at the scale cursor: lane l loads word l%8 of
    // group rows glo + l/8 and glo + 4 + l/8 (16 columns of f16 = 8 words)
    auto scale_fetch = [&](uint32_t &r0, uint32_t &r1) {
      r0 = r1 = 0;
      if (sc.si >= nseg) return;
      const WlSeg &sg = segs[sc.si];
      const WlItem &it = p.items[sg.item];
      if (it.kind == kWlQ4) {
        const int nb = it.nb0 + sg.u0 + first_of(sg, cw) + sc.j * kWlWarps;
        const int glo = sc.st * 8 / it.gk, ng = 8 / it.gk;
        const uint8_t *row = static_cast<const uint8_t *>(it.b_scale) +
                             ((size_t)glo * it.N + (size_t)nb * 16) * 2 + (lane & 7) * 4;
        const int q = lane >> 3;
        if (q < ng) r0 = ldg_stream_u32(row + (size_t)q * it.N * 2);
        if (q + 4 < ng) r1 = ldg_stream_u32(row + (size_t)(q + 4) * it.N * 2);
      }
      advance(sc, segs, nseg, cw);
    };

    // the weights never come from earlier kernels: fill the ring first
    while (issued < S && ic.si < nseg) issue();
    uint32_t sa0, sa1, sb0, sb1;
    scale_fetch(sa0, sa1);
    scale_fetch(sb0, sb1);
    pdl_wait();  // prep sources and GEMM outputs are ordered after earlier kernels

    bool ok = true;
    int g = 0;
    for (int si = 0; si < nseg && ok; si++) {
      const WlSeg sg = segs[si];
      const WlItem &it = p.items[sg.item];
      const int first = first_of(sg, cw), n_my = count_of(sg, cw);
      if (sg.kind == kWlPrep) {
        if (n_my == 0) continue;
        if (lane == 0) ok = wl_wait_item(p, it.deps[0]) && wl_wait_item(p, it.deps[1]);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
        for (int j = 0; j < n_my; j++) prep_row(it, sg.u0 + first + j * kWlWarps, p.M, lane);
        wl_signal(p, sg.item, (unsigned)n_my, lane);
        continue;
      }
      const int b = g % p.n_abuf;
      const uint32_t fpar = (uint32_t)((g / p.n_abuf) & 1);
      g++;
      ok = __all_sync(0xffffffffu, wl_wait(&s_full[b], fpar, p));
      if (!ok) break;
      const uint32_t ab = abuf0 + (uint32_t)(b * p.abuf_bytes);
      const bool q4 = it.kind == kWlQ4;
      const int T = q4 ? 8 : 4;
      for (int j = 0; j < n_my && ok; j++) {
        const int nb = it.nb0 + sg.u0 + first + j * kWlWarps;
        float cf[MT][4];
        int32_t acc[MT][4];
#pragma unroll
        for (int mt = 0; mt < MT; mt++)
#pragma unroll
          for (int i = 0; i < 4; i++) {
            cf[mt][i] = 0.0f;
            acc[mt][i] = 0;
          }
        float bs0 = 0.0f, bs1 = 0.0f;  // int8 per-channel scales of columns g8, g8 + 8
        if (!q4) {
          const float *bsp = static_cast<const float *>(it.b_scale) + nb * 16 + L.g8;
          bs0 = bsp[0];
          bs1 = bsp[8];
        }
        for (int st = 0; st < sg.nst; st++) {
          const uint32_t c0 = sa0, c1 = sa1;
          sa0 = sb0;
          sa1 = sb1;
          scale_fetch(sb0, sb1);
          const int slot = consumed % S;
          ok = __all_sync(0xffffffffu, wl_wait(&bars[slot], (uint32_t)((consumed / S) & 1), p));
          if (!ok) break;
          const uint32_t stg = ring + slot * kWlStage;
          const uint32_t abs_ = ab + (uint32_t)(st * T * MT * 512);
          if (q4) q4_stage_gk<MT>(it.gk, stg, abs_, L, c0, c1, cf);
          else q8_stage<MT>(stg, abs_, L, acc);
          __syncwarp();
          fence_proxy_async_smem();  // this warp's reads of the slot precede its refill
          consumed++;
          if (ic.si < nseg) issue();
        }
        if (!ok) break;
#pragma unroll
        for (int mt = 0; mt < MT; mt++)
#pragma unroll
          for (int i = 0; i < 4; i++) {
            const int m = mt * 8 + 2 * L.tig + (i & 1);
            const int n = nb * 16 + L.g8 + (i >= 2 ? 8 : 0);
            if (m >= p.M) continue;
            const float as = s_as[b][m];
            it.C[(size_t)m * it.ldc + (n - it.c_col0)] =
                q4 ? __fmul_rn(cf[mt][i], as)
                   : __fmul_rn(__int2float_rn(acc[mt][i]), __fmul_rn(i < 2 ? bs0 : bs1, as));
          }
      }
      if (!ok) break;
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(
                                      tc::smem_u32(&s_empty[b]))
                                  : "memory");
      if (n_my > 0) wl_signal(p, sg.item, (unsigned)n_my, lane);
    }
    if (!ok) {
      if (lane == 0) wl_fail(p, 5);
      // weight stages still in flight land before the CTA exits
      for (int k = consumed; k < issued; k++)
        tc::mbar_wait(&bars[k % S], (uint32_t)((k / S) & 1));
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
size_t worklist_smem(int n_abuf, int abuf_bytes, int stages) {
  return 1024 + (size_t)n_abuf * abuf_bytes + (size_t)kWlWarps * stages * kWlStage;
}

int worklist_consumers() { return kWlWarps; }

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
  // ---- shared memory: activation buffers and the weight rings
  int max_kb = 0;
  for (const WlItem &it : items)
    if (it.kind != kWlPrep) max_kb = std::max(max_kb, it.K / 64);
  pl.abuf_bytes = std::max(1024, (pl.MT * 512 * max_kb + 1023) / 1024 * 1024);
  const size_t limit = smem_optin + 1024 - (size_t)wl_static_smem(pl.MT) - 256;
  pl.n_abuf = 0;
  for (int nb = 2; nb >= 1 && !pl.n_abuf; nb--) {
    for (int s = kWlMaxStages; s >= (nb == 2 ? 3 : 2); s--)
      if (worklist_smem(nb, pl.abuf_bytes, s) <= limit) {
        pl.n_abuf = nb;
        pl.stages = s;
        break;
      }
  }
  if (!pl.n_abuf) return "the activations of the widest item do not fit in shared memory";
  pl.smem = worklist_smem(pl.n_abuf, pl.abuf_bytes, pl.stages);

  // ---- levels: one more than the deepest dependency
  std::vector<int> level(n, 0);
  int nlev = 0;
  for (int i = 0; i < n; i++) {
    for (int d : items[i].deps)
      if (d >= 0) level[i] = std::max(level[i], level[d] + 1);
    nlev = std::max(nlev, level[i] + 1);
  }
  // ---- segments per CTA, level by level
  const int G = num_sms;
  std::vector<std::vector<WlSeg>> cta(G);
  std::vector<int> base(G, 0);
  int rr = 0;  // round-robin position of prep rows
  auto push = [&](int c, int item, int u0, int u1) {
    const WlItem &it = items[item];
    WlSeg sg{};
    sg.item = item;
    sg.u0 = u0;
    sg.u1 = u1;
    sg.base = base[c];
    sg.kind = it.kind;
    sg.nst = it.kind == kWlQ4 ? it.K / 512 : (it.kind == kWlQ8 ? it.K / 256 : 0);
    base[c] = (base[c] + (u1 - u0)) % kWlWarps;
    cta[c].push_back(sg);
  };
  for (int lv = 0; lv < nlev; lv++) {
    // GEMM units of the level, flattened in list order, split by weight bytes
    double total = 0;
    for (int i = 0; i < n; i++)
      if (level[i] == lv && items[i].kind != kWlPrep)
        total += (double)items[i].units * (items[i].kind == kWlQ4 ? items[i].K / 512 : items[i].K / 256);
    double acc = 0;
    for (int i = 0; i < n; i++) {
      if (level[i] != lv) continue;
      WlItem &it = items[i];
      if (it.kind == kWlPrep) {
        for (int u = 0; u < it.units; u++) {
          push(rr % G, i, u, u + 1);
          rr++;
        }
        continue;
      }
      const double cost = it.kind == kWlQ4 ? it.K / 512 : it.K / 256;
      int u = 0;
      while (u < it.units) {
        // the CTA whose share holds this unit's midpoint, and how far its share goes
        const int c = std::min(G - 1, (int)((acc + 0.5 * cost) * G / total));
        const double end = (double)(c + 1) * total / G;
        int u1 = u + 1;
        while (u1 < it.units && acc + (u1 - u + 0.5) * cost < end) u1++;
        push(c, i, u, u1);
        acc += (u1 - u) * cost;
        u = u1;
      }
    }
  }
  pl.seg_off.assign(G + 1, 0);
  pl.segs.clear();
  for (int c = 0; c < G; c++) {
    pl.seg_off[c] = (int)pl.segs.size();
    pl.segs.insert(pl.segs.end(), cta[c].begin(), cta[c].end());
  }
  pl.seg_off[G] = (int)pl.segs.size();
  return nullptr;
}

cudaError_t launch_worklist(const WlParams &p, const WlPlan &pl, bool pdl, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.grid);
  cfg.blockDim = dim3((kWlWarps + 1) * 32);
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
