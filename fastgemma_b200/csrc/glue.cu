// Decode-chain glue and the int8-KV attention on the device: the operations
// between the GEMMs of fgm-core's forward pass (forward.rs:469-654), as the
// reference's fgm-kernels implements them (crates/fgm-kernels/csrc/ops.c).
//
// The reference runs these 16 floats at a time (AVX-512) and finishes a
// length that is not a multiple of 16 with scalar libm code.  The kernels
// below reproduce the vector arithmetic element by element in the same order
// -- its Cephes-style exp (ops.c:21-39), its 16-lane accumulations and their
// reduction tree, every multiply / add / fused multiply-add as the reference
// rounds it (explicit _rn intrinsics, no contraction) -- so their outputs are
// bit-identical to the reference wherever it does not call libm.  The libm
// pieces (tails past the last multiple of 16, rope's cosf / sinf, the
// softmax tail's expf) are evaluated in double precision and rounded once,
// which agrees with a correctly rounded libm; they are checked to a tolerance.
//
// Attention (ops.c:378-640) is one cluster of CTAs per (query row, KV head),
// split by cache slot: the per-head int8 quantisation of Q, exact int8 Q.K
// dot products and the exact P.V against the slot-interleaved V cache
// (signed V bytes times the unsigned bytes of the 16-bit split weights) on
// the tensor cores, the softmax with the reference's lane order for the sum.
// Integer sums are exact in any order; every float step follows the
// reference's order, so the output is bit-identical.

#include <cooperative_groups.h>

#include "fgm_common.cuh"
#include "fgm_internal.h"

namespace cg = cooperative_groups;

namespace fgm {

namespace {

// One lane of ops.c:21-39: clamp to [-88, 88], n = rint(x log2 e),
// z = x - n ln2 in two parts, degree-5 polynomial, times 2^n.
__device__ __forceinline__ float exp_lane(float x) {
  x = fmaxf(x, -88.0f);
  x = fminf(x, 88.0f);
  const float fx = rintf(__fmul_rn(x, 1.44269504088896341f));
  float z = __fmaf_rn(-fx, 0.693359375f, x);
  z = __fmaf_rn(-fx, -2.12194440e-4f, z);
  float y = 1.9875691500E-4f;
  y = __fmaf_rn(y, z, 1.3981999507E-3f);
  y = __fmaf_rn(y, z, 8.3334519073E-3f);
  y = __fmaf_rn(y, z, 4.1665795894E-2f);
  y = __fmaf_rn(y, z, 1.6666665459E-1f);
  y = __fmaf_rn(y, z, 5.0000001201E-1f);
  y = __fmaf_rn(y, __fmul_rn(z, z), z);
  y = __fadd_rn(y, 1.0f);
  const int n = (int)fx;  // fx is integral, in [-127, 127]
  return __fmul_rn(y, __int_as_float((n + 127) << 23));
}

// ops.c:96-107, one lane.
__device__ __forceinline__ float gelu_lane(float x) {
  const float x3 = __fmul_rn(__fmul_rn(x, x), x);
  const float u = __fmul_rn(0.7978845608028654f, __fmaf_rn(0.044715f, x3, x));
  const float e = exp_lane(__fadd_rn(u, u));
  const float t = __fsub_rn(1.0f, __fdiv_rn(2.0f, __fadd_rn(e, 1.0f)));
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, t));
}

// The scalar tail of ops.c:119-131 (libm tanhf).
__device__ __forceinline__ float gelu_tail(float v) {
  const float in = __fmul_rn(0.7978845608028654f,
                             __fadd_rn(v, __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, v), v), v)));
  const float th = (float)tanh((double)in);
  return __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, th));
}

// _mm512_reduce_add_ps as the reference's build lowers it: lanes (i, i+8),
// then (i, i+4), then (i, i+2), then the last pair.
__device__ __forceinline__ float reduce16(const float *a) {
  float t8[8], t4[4];
#pragma unroll
  for (int i = 0; i < 8; i++) t8[i] = __fadd_rn(a[i], a[i + 8]);
#pragma unroll
  for (int i = 0; i < 4; i++) t4[i] = __fadd_rn(t8[i], t8[i + 4]);
  return __fadd_rn(__fadd_rn(t4[0], t4[2]), __fadd_rn(t4[1], t4[3]));
}

// One of the reference's 16 accumulator lanes over a row in shared memory:
// acc = fmaf(x[i], x[i], acc) for i = lane, lane + 16, ... < full, in that
// order.  Loads go out eight at a time so the chain waits on FMAs only.
__device__ __forceinline__ float lane_sumsq(const float *x, int lane, int full) {
  float acc = 0.0f;
  int i = lane;
  for (; i + 16 * 7 < full; i += 16 * 8) {
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; k++) v[k] = x[i + 16 * k];
#pragma unroll
    for (int k = 0; k < 8; k++) acc = __fmaf_rn(v[k], v[k], acc);
  }
  for (; i < full; i += 16) acc = __fmaf_rn(x[i], x[i], acc);
  return acc;
}

constexpr int kGlueThreads = 256;

// ops.c:59-92, one row per CTA.  The row goes through shared memory; 16
// threads keep the reference's 16 accumulator lanes (fmaf chains over the
// full chunks, in order), thread 0 reduces them and adds the tail.
__global__ void __launch_bounds__(kGlueThreads) rmsnorm_kernel(float *out, const float *x,
                                                              const float *w, int n, float eps) {
  extern __shared__ float xs[];
  __shared__ float lanes[16];
  __shared__ float s_inv;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const float *xr = x + (size_t)blockIdx.x * n;
  float *orow = out + (size_t)blockIdx.x * n;
  for (int i = threadIdx.x; i < n; i += blockDim.x) xs[i] = xr[i];
  __syncthreads();
  const int full = n & ~15;
  if (threadIdx.x < 16) {
    lanes[threadIdx.x] = lane_sumsq(xs, threadIdx.x, full);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float ss = reduce16(lanes);
    for (int i = full; i < n; i++) ss = __fmaf_rn(xs[i], xs[i], ss);
    s_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
  }
  __syncthreads();
  const float inv = s_inv;
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    orow[i] = w ? __fmul_rn(__fmul_rn(xs[i], inv), w[i]) : __fmul_rn(xs[i], inv);
}

// ops.c:119-131 over rows of n (each row's tail is the reference's scalar tail).
__global__ void gelu_mul_kernel(float *out, const float *gate, const float *up, int n, size_t total) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int full = n & ~15;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const int col = (int)(i % (size_t)n);
    out[i] = __fmul_rn(col < full ? gelu_lane(gate[i]) : gelu_tail(gate[i]), up[i]);
  }
}

// ops.c:317-337: op 0 add, 1 mul, 2 scale by s.
__global__ void elementwise_kernel(float *a, const float *b, float s, size_t n, int op) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    a[i] = op == 0 ? __fadd_rn(a[i], b[i]) : op == 1 ? __fmul_rn(a[i], b[i]) : __fmul_rn(a[i], s);
}

// ops.c:340-352 over rows of n.
__global__ void softcap_kernel(float *x, int n, size_t total, float cap) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const float ci = __fdiv_rn(1.0f, cap);
  const int full = n & ~15;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const float v = x[i];
    if ((int)(i % (size_t)n) < full) {
      const float u = __fmul_rn(v, ci);
      const float e = exp_lane(__fadd_rn(u, u));
      x[i] = __fmul_rn(cap, __fsub_rn(1.0f, __fdiv_rn(2.0f, __fadd_rn(e, 1.0f))));
    } else {
      x[i] = __fmul_rn(cap, (float)tanh((double)__fdiv_rn(v, cap)));
    }
  }
}

// Rope's cos and sin of angle pos * inv_freq[j]: from the caller's host
// table (cs[pos][head_dim]: cos in [0, half), sin in [half, 2 half), the
// reference's own libm values) when the position is inside it, else
// evaluated in double precision and rounded once.
__device__ __forceinline__ void rope_cs(const float *inv_freq, const float *tab, int positions,
                                        int half, int pos, int j, float &c, float &s) {
  if (tab && pos >= 0 && pos < positions) {
    const float *t = tab + (size_t)pos * 2 * half;
    c = t[j];
    s = t[half + j];
  } else {
    const float a = __fmul_rn((float)pos, inv_freq[j]);
    c = (float)cos((double)a);
    s = (float)sin((double)a);
  }
}

// ops.c:135-147 for `rows` rows (row r at x + r*x_ld, position pos[r]).  The
// reference's build fuses each product pair into one rounding.
__global__ void rope_kernel(float *x, int x_ld, int n_heads, int head_dim, const float *inv_freq,
                            const float *tab, int positions, const int *pos) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int h = head_dim / 2, r = blockIdx.y;
  float *xr = x + (size_t)r * x_ld;
  for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < n_heads * h;
       idx += gridDim.x * blockDim.x) {
    const int hh = idx / h, j = idx % h;
    float c, s;
    rope_cs(inv_freq, tab, positions, h, pos[r], j, c, s);
    float *p = xr + (size_t)hh * head_dim;
    const float lo = p[j], hi = p[j + h];
    p[j] = __fmaf_rn(lo, c, -__fmul_rn(hi, s));
    p[j + h] = __fmaf_rn(hi, c, __fmul_rn(lo, s));
  }
}

// ops.c:653-660 for `rows` caches (row r: cache vt + r*vt_stride, source
// src + r*src_ld): one int8 V row into the slot-interleaved layout.
__global__ void store_v_t_kernel(int8_t *vt, size_t vt_stride, const int8_t *src, int src_ld, int n,
                                 int slot) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int r = blockIdx.y;
  int8_t *dst = vt + (size_t)r * vt_stride + (size_t)(slot >> 2) * n * 4 + (slot & 3);
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < n; j += gridDim.x * blockDim.x)
    dst[(size_t)j * 4] = src[(size_t)r * src_ld + j];
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float u = __shfl_xor_sync(0xffffffffu, v, o);
    v = u > v ? u : v;
  }
  return v;
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src) : "memory");
}

__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
  const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(d), "l"(src) : "memory");
}

__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// D += A(16x32 s8, row) * B(32x8 u8, col), int32 accumulate: signed V bytes
// times unsigned weight bytes.
__device__ __forceinline__ void mma_s8u8_m16n8k32(int32_t (&d)[4], uint32_t a0, uint32_t a1,
                                                  uint32_t a2, uint32_t a3, uint32_t b0,
                                                  uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t lds32(const void *p) {
  return *reinterpret_cast<const uint32_t *>(p);
}

// ops.c:378-640 for one query row and one KV head with the G query heads
// that share it, split over a cluster of C CTAs by cache slot: CTA `rank`
// owns the slots [wbase + rank*cs, +cs) (cs = 4*gchunk, whole V groups) and
// scores, exponentiates, weights and multiplies the window positions held
// there.  Everything that needs a fixed order stays exact: the softmax max
// and the weight max are order-free, every CTA runs the reference's 16 lane
// sums over the whole window itself (gathering the other CTAs'
// exponentials through distributed shared memory, window by window), and
// the integer sums -- Q.K on the tensor cores (mma s8 x s8), P.V likewise
// (s8 V x u8 weight bytes) -- meet by integer atomics in the CTA that owns
// each output dimension.  Shared memory (offsets from the host): Q as int8
// [GM][hd], K and V scales [cs], a K stage [kp][hd + 16], a V stage
// [vgp][hd * 4 + 32] (slot-interleaved), the exponentials [GM][cs], the
// gather window [GM][win], the stage's weight bytes [2 GM][vgp * 4 + 16]
// (column 2h: high bytes of head h, 2h + 1: low bytes) and the int32
// accumulators [2 GM][hd].  Row paddings keep the fragment loads free of
// bank conflicts.
//
// ONE (the whole window fits one gather, the usual decode case): after the
// gather every CTA holds all exponentials, so it computes the weight max and
// all weight bytes itself and multiplies every slot against its own
// head_dim / C output dimensions -- V staged as [group][its dims + padding],
// the V scales of all slots, the weights and then the P.V partial sums in
// the K stage, results stored directly.  That drops the weight-max exchange
// and the integer atomics; the last cluster barrier is split (arrive after
// the gather, wait at exit) so that no CTA leaves while a peer may still
// read its exponentials.  With fewer heads than warps, the spare warps issue
// the V copies while the others quantise Q.
template <int GM, bool ONE>
__global__ void __launch_bounds__(kGlueThreads) attend_q8_kernel(const AttnParams p) {
  constexpr int nt = kGlueThreads, nw = kGlueThreads / 32;
  constexpr int kTiles = (512 / 16) * ((2 * GM + 7) / 8) / nw;  // P.V tiles per warp, at most
  cg::cluster_group cluster = cg::this_cluster();
  extern __shared__ __align__(16) uint8_t sm[];
  __shared__ float s_qscale[GM], s_lmax[GM], s_mx[GM], s_inv[GM], s_lwmax[GM], s_wmax[GM],
      s_wqs[GM], s_wqi[GM];
  __shared__ float s_lanes[GM][16];
  __shared__ float s_red[nw][GM];
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int G = p.n_heads / p.kv_heads, C = p.cluster;
  const int rank = (int)cluster.block_rank();
  const int kvh = blockIdx.x / C, r = blockIdx.y;
  const int hd = p.head_dim, kvd = p.kv_heads * hd, n = p.end - p.start;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, gid = lane >> 2, tig = lane & 3;
  const int cs = p.gchunk * 4, kld = hd + 16, vld = hd * 4 + 32, kp = p.kp, vg = p.vg;
  const int wld = p.vgp * 4 + 16, win = p.win;
  const int S0 = min(p.wbase + p.wslots, p.wbase + rank * cs);
  const int ns = min(p.wbase + p.wslots, S0 + cs) - S0;  // a multiple of 4
  const int tb = p.ring ? p.start - p.start % p.ring : 0;
  int8_t *qq = reinterpret_cast<int8_t *>(sm);
  float *ksm = reinterpret_cast<float *>(sm + p.off_ks);
  float *vsm = ksm + cs;
  int8_t *kst = reinterpret_cast<int8_t *>(sm + p.off_k);
  int8_t *vst = reinterpret_cast<int8_t *>(sm + p.off_v);
  float *ev = reinterpret_cast<float *>(sm + p.off_e);
  float *wbuf = reinterpret_cast<float *>(sm + p.off_win);
  uint8_t *wst = sm + p.off_w;
  int *acc = reinterpret_cast<int *>(sm + p.off_acc);
  const int8_t *kc = p.kc + (size_t)r * p.kc_stride + (size_t)kvh * hd;
  const float *ks = p.ks + (size_t)r * p.ks_stride;
  const int8_t *vt = p.vt + (size_t)r * p.vt_stride + (size_t)kvh * hd * 4;
  const float *vs = p.vs + (size_t)r * p.vs_stride;
  const int full = n & ~15;
  const int dper = hd / C, d0 = rank * dper;  // ONE: this CTA's output dimensions
  const int vldo = dper * 4 + 32;             // ONE: bytes per V group row (padded)
  float *vsa = reinterpret_cast<float *>(sm + p.off_vsa);  // ONE: V scales of all slots

  // window position held by cache slot s, or -1
  auto pos_of = [&](int s) -> int {
    if (p.ring) {
      if (s >= p.ring) return -1;
      int t = tb + s;
      if (t < p.start) t += p.ring;
      return t < p.end ? t - p.start : -1;
    }
    return (s >= p.start && s < p.end) ? s - p.start : -1;
  };
  const int wdt = p.vec16 ? 16 : 4;
  auto load_k = [&](int sa, int sb) {  // this CTA's slots [sa, sb), rows of this KV head
    const int per = hd / wdt, rpp = nt / per, piece = tid % per;
    if (tid < rpp * per)
      for (int j = sa + tid / per; j < sb; j += rpp) {
        if (pos_of(S0 + j) < 0) continue;
        int8_t *dst = kst + (j - sa) * kld + piece * wdt;
        const int8_t *src = kc + (size_t)(S0 + j) * kvd + piece * wdt;
        if (p.vec16)
          cp_async16(dst, src);
        else
          cp_async4(dst, src);
      }
    cp_async_commit();
  };
  auto load_v = [&](int ga, int gb) {  // this CTA's slot groups [ga, gb)
    const int per = hd * 4 / wdt;
    const int8_t *src = vt + (size_t)(S0 / 4) * kvd * 4;
    auto copy = [&](int g, int piece) {
      int8_t *dst = vst + (g - ga) * vld + piece * wdt;
      const int8_t *s = src + (size_t)g * kvd * 4 + piece * wdt;
      if (p.vec16)
        cp_async16(dst, s);
      else
        cp_async4(dst, s);
    };
    if (per <= nt) {
      const int rpp = nt / per;
      if (tid < rpp * per)
        for (int g = ga + tid / per; g < gb; g += rpp) copy(g, tid % per);
    } else {
      for (int g = ga; g < gb; g++)
        for (int piece = tid; piece < per; piece += nt) copy(g, piece);
    }
    cp_async_commit();
  };

  // ONE: every slot group of this KV head, this CTA's dims
  // by threads [t0, t0 + nthr); every thread commits (equal group counts)
  auto load_v_dims = [&](int t0, int nthr) {
    const int per = dper * 4 / wdt, t = tid - t0;
    const int8_t *src = vt + (size_t)(p.wbase / 4) * kvd * 4 + (size_t)d0 * 4;
    if (t >= 0 && t < nthr) {
      if (per <= nthr) {
        const int gpp = nthr / per, piece = t % per;
        if (t < gpp * per)
          for (int g = t / per; g < p.wslots / 4; g += gpp) {
            int8_t *dst = vst + g * vldo + piece * wdt;
            const int8_t *sp = src + (size_t)g * kvd * 4 + piece * wdt;
            if (p.vec16)
              cp_async16(dst, sp);
            else
              cp_async4(dst, sp);
          }
      } else {
        for (int g = 0; g < p.wslots / 4; g++)
          for (int piece = t; piece < per; piece += nthr) {
            int8_t *dst = vst + g * vldo + piece * wdt;
            const int8_t *sp = src + (size_t)g * kvd * 4 + piece * wdt;
            if (p.vec16)
              cp_async16(dst, sp);
            else
              cp_async4(dst, sp);
          }
      }
    }
    cp_async_commit();
  };
  // ONE: with fewer heads than warps the spare warps issue the V copies
  // while the others quantise Q
  const bool v_late = ONE && G < nw;

  if constexpr (!ONE)
    for (int i = tid; i < GM * 2 * hd; i += nt) acc[i] = 0;
  for (int j = tid; j < ns; j += nt)
    if (pos_of(S0 + j) >= 0) {
      cp_async4(ksm + j, ks + S0 + j);
      cp_async4(vsm + j, vs + S0 + j);
    }
  if constexpr (ONE)
    for (int s = tid; s < p.wslots; s += nt)
      if (pos_of(p.wbase + s) >= 0) cp_async4(vsa + s, vs + p.wbase + s);
  load_k(0, min(ns, kp));  // commits the scales with the first K stage
  if constexpr (ONE) {
    if (!v_late) load_v_dims(0, nt);
  } else {
    load_v(0, min(ns / 4, vg));
  }

  // ---- Q per head: int8 with one scale (ops.c:412-431)
  for (int h = warp; h < G; h += nw) {
    const float *qh = p.q + (size_t)r * p.q_ld + (size_t)(kvh * G + h) * hd;
    float qv[16];
    float a = 0.0f;
#pragma unroll
    for (int k = 0; k < 16; k++) {
      qv[k] = lane + 32 * k < hd ? qh[lane + 32 * k] : 0.0f;
      const float v = fabsf(qv[k]);
      a = v > a ? v : a;
    }
    const float qamax = warp_max(a);
    const float qinv = qamax > 0.0f ? __fdiv_rn(127.0f, qamax) : 0.0f;
#pragma unroll
    for (int k = 0; k < 16; k++)
      if (lane + 32 * k < hd) {
        const int v = __float2int_rn(__fmul_rn(qv[k], qinv));
        qq[h * hd + lane + 32 * k] = (int8_t)(v > 127 ? 127 : (v < -127 ? -127 : v));
      }
    if (lane == 0) s_qscale[h] = __fdiv_rn(qamax, 127.0f);
  }
  if (v_late) load_v_dims(G * 32, nt - G * 32);

  // ---- scores: exact int8 dots (ops.c:432-474), slots x heads on the
  // tensor cores; an empty slot scores -inf here and weighs 0 below
  for (int sa = 0; sa < ns; sa += kp) {
    const int sb = min(ns, sa + kp), rows = sb - sa;
    if (sa) {
      load_k(sa, sb);
      cp_async_wait<0>();
    } else {
      cp_async_wait<1>();
    }
    __syncthreads();
    const int mt = (rows + 15) >> 4, tiles = mt * ((G + 7) >> 3);
    for (int tile = warp; tile < tiles; tile += nw) {
      const int m0 = (tile % mt) * 16, n0 = (tile / mt) * 8;
      const int8_t *ar = kst + (m0 + gid) * kld + tig * 4;
      const int8_t *br = qq + min(n0 + gid, G - 1) * hd + tig * 4;
      int32_t d[4] = {0, 0, 0, 0};
      for (int kb = 0; kb < hd; kb += 32)
        mma_s8_m16n8k32(d, lds32(ar + kb), lds32(ar + 8 * kld + kb), lds32(ar + kb + 16),
                        lds32(ar + 8 * kld + kb + 16), lds32(br + kb), lds32(br + kb + 16));
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const int row = m0 + gid + (e >> 1) * 8, h = n0 + 2 * tig + (e & 1), j = sa + row;
        if (row < rows && h < G)
          ev[h * cs + j] = pos_of(S0 + j) < 0
                               ? -INFINITY
                               : __fmul_rn(__fmul_rn((float)d[e], s_qscale[h]), ksm[j]);
      }
    }
    __syncthreads();
  }
  for (int h = warp; h < G; h += nw) {
    float m = -INFINITY;
    for (int j = lane; j < ns; j += 32) {
      const float v = ev[h * cs + j];
      m = v > m ? v : m;
    }
    m = warp_max(m);
    if (lane == 0) s_lmax[h] = m;
  }
  cluster.sync();
  if (tid < G) {
    float v[8];
#pragma unroll
    for (int c = 0; c < 8; c++) v[c] = c < C ? cluster.map_shared_rank(s_lmax, c)[tid] : -INFINITY;
    float m = v[0];
#pragma unroll
    for (int c = 1; c < 8; c++) m = v[c] > m ? v[c] : m;
    s_mx[tid] = m;
  }
  __syncthreads();

  // ---- exponentials: the reference's exp lanes over the 16-position
  // chunks, libm (here: double, rounded once) on the tail
  for (int idx = tid; idx < G * ns; idx += nt) {
    const int h = idx / ns, j = idx - h * ns;
    const int u = pos_of(S0 + j);
    float *e = ev + h * cs + j;
    if (u < 0) {
      *e = 0.0f;
    } else {
      const float d = __fsub_rn(*e, s_mx[h]);
      *e = u < full ? exp_lane(d) : (float)exp((double)d);
    }
  }
  cluster.sync();

  // ---- the sum in the reference's order: 16 lanes over the full chunks,
  // reduced, then the tail.  Windows of `win` positions (a multiple of 16)
  // are gathered from the owning CTAs first.
  {
    float l = 0.0f;
    const int h = tid >> 4, ln = tid & 15;
    for (int w0 = 0; w0 < n; w0 += win) {
      const int wn = min(n, w0 + win) - w0;
      int s0 = p.start + w0;
      if (p.ring) s0 %= p.ring;
      s0 -= p.wbase;
      __syncthreads();
      constexpr int kB = GM <= 4 ? 4 : (GM <= 8 ? 2 : 1);  // positions a thread has in flight
      if (!p.ring && (p.start & 3) == 0) {
        // slots run with positions from a 4-aligned start: four positions are
        // four slots of one owner, moved as one 16-byte load (any values past
        // the window end are exponentials of empty slots, 0, never read)
        for (int i = 4 * tid; i < wn; i += 4 * nt) {
          const int sl = s0 + i, c = sl / cs;
          const float *pe = cluster.map_shared_rank(ev, c) + (sl - c * cs);
          float4 v[GM];
#pragma unroll
          for (int hh = 0; hh < GM; hh++)
            if (hh < G) v[hh] = *reinterpret_cast<const float4 *>(pe + hh * cs);
#pragma unroll
          for (int hh = 0; hh < GM; hh++)
            if (hh < G) *reinterpret_cast<float4 *>(wbuf + hh * win + i) = v[hh];
        }
      } else
      for (int i0 = 0; i0 < wn; i0 += kB * nt) {
        float v[kB][GM];
#pragma unroll
        for (int k = 0; k < kB; k++) {
          const int i = i0 + k * nt + tid;
          if (i < wn) {
            int s = s0 + i;
            if (p.ring && s >= p.ring) s -= p.ring;
            const int c = s / cs;
            const float *pe = cluster.map_shared_rank(ev, c) + (s - c * cs);
#pragma unroll
            for (int hh = 0; hh < GM; hh++) v[k][hh] = hh < G ? pe[hh * cs] : 0.0f;
          }
        }
#pragma unroll
        for (int k = 0; k < kB; k++) {
          const int i = i0 + k * nt + tid;
          if (i < wn)
#pragma unroll
            for (int hh = 0; hh < GM; hh++)
              if (hh < G) wbuf[hh * win + i] = v[k][hh];
        }
      }
      __syncthreads();
      if constexpr (ONE)  // the last read of another CTA's shared memory
        asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
      if (tid < G * 16)
        for (int u = w0 + ln; u < min(w0 + wn, full); u += 16)
          l = __fadd_rn(l, wbuf[h * win + u - w0]);
    }
    if (tid < G * 16) s_lanes[h][ln] = l;
    __syncthreads();
    if (tid < G) {
      const int wl = ((n - 1) / win) * win;  // the last window holds the tail
      float sum = reduce16(s_lanes[tid]);
      for (int u = full; u < n; u++) sum = __fadd_rn(sum, wbuf[tid * win + u - wl]);
      s_inv[tid] = __fdiv_rn(1.0f, sum);
    }
    __syncthreads();
  }

  if constexpr (ONE) {
    // ---- weights of every slot, their max per head, then P.V against this
    // CTA's dimensions (ops.c:560-625)
    cp_async_wait<0>();  // V scales and V (a CTA without slots never waited)
    __syncthreads();
    // weights per (head, group of 4 slots) into wf (the K stage is free now);
    // an empty slot weighs 0
    const int kpad = (p.wslots + 31) & ~31, ngr = kpad >> 2;
    float *wf = reinterpret_cast<float *>(kst);  // [G][kpad]
    {
      float wl[GM];
#pragma unroll
      for (int h = 0; h < GM; h++) wl[h] = 0.0f;
      for (int g = tid; g < ngr; g += nt) {
        int u[4];
        float vsv[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const int sl = 4 * g + j;
          u[j] = sl < p.wslots ? pos_of(p.wbase + sl) : -1;
          vsv[j] = u[j] < 0 ? 0.0f : vsa[sl];
        }
#pragma unroll
        for (int h = 0; h < GM; h++)
          if (h < G) {
            float w4[4];
#pragma unroll
            for (int j = 0; j < 4; j++) {
              w4[j] = u[j] < 0 ? 0.0f
                               : __fmul_rn(__fmul_rn(wbuf[h * win + u[j]], s_inv[h]), vsv[j]);
              wl[h] = w4[j] > wl[h] ? w4[j] : wl[h];
            }
            *reinterpret_cast<float4 *>(wf + h * kpad + 4 * g) =
                make_float4(w4[0], w4[1], w4[2], w4[3]);
          }
      }
#pragma unroll
      for (int h = 0; h < GM; h++) wl[h] = warp_max(wl[h]);
      if (lane == 0)
#pragma unroll
        for (int h = 0; h < GM; h++) s_red[warp][h] = wl[h];
    }
    __syncthreads();
    if (tid < G) {
      float m = s_red[0][tid];
      for (int w = 1; w < nw; w++) m = s_red[w][tid] > m ? s_red[w][tid] : m;
      s_wmax[tid] = m;
      s_wqs[tid] = __fdiv_rn(m, 65535.0f);
      s_wqi[tid] = m > 0.0f ? __fdiv_rn(65535.0f, m) : 0.0f;
    }
    __syncthreads();
    // 16-bit weights of their max, high and low bytes packed four slots a word
#pragma unroll
    for (int h = 0; h < GM; h++)
      if (h < G) {
        const bool live = s_wmax[h] > 0.0f;
        const float wqi = s_wqi[h];
        for (int g = tid; g < ngr; g += nt) {
          const float4 w4 = *reinterpret_cast<const float4 *>(wf + h * kpad + 4 * g);
          const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
          uint32_t hi = 0, lo = 0;
#pragma unroll
          for (int j = 0; j < 4; j++) {
            int iw = 0;
            if (live) {
              iw = (int)__fadd_rn(__fmul_rn(wv[j], wqi), 0.5f);
              iw = iw > 65535 ? 65535 : (iw < 0 ? 0 : iw);
            }
            hi |= (uint32_t)(iw >> 8) << (8 * j);
            lo |= (uint32_t)(iw & 255) << (8 * j);
          }
          *reinterpret_cast<uint32_t *>(wst + (2 * h) * wld + 4 * g) = hi;
          *reinterpret_cast<uint32_t *>(wst + (2 * h + 1) * wld + 4 * g) = lo;
        }
      }
    __syncthreads();
    // tiles: 16 dims x 8 columns (head h: columns 2h, 2h + 1 = high, low
    // bytes); the k steps of a tile split over the warps that share it,
    // partial sums added in shared memory (integers: any order)
    const int pm = dper >> 4, pn = (2 * G + 7) >> 3, tiles = pm * pn;
    const int split = nw / tiles > 0 ? nw / tiles : 1, ksteps = kpad >> 5;
    int *part = reinterpret_cast<int *>(kst);  // the K stage is free now
    for (int tw = warp; tw < tiles * split; tw += nw) {
      const int tile = tw % tiles, sp = tw / tiles;
      const int m0 = (tile % pm) * 16, n0 = (tile / pm) * 8;
      const int8_t *ar = vst + tig * vldo + (m0 + gid) * 4;
      const uint8_t *br = wst + min(n0 + gid, 2 * G - 1) * wld + tig * 4;
      int32_t d[4] = {0, 0, 0, 0};
      for (int ks = sp; ks < ksteps; ks += split) {
        const int8_t *a = ar + ks * 8 * vldo;
        mma_s8u8_m16n8k32(d, lds32(a), lds32(a + 32), lds32(a + 4 * vldo),
                          lds32(a + 4 * vldo + 32), lds32(br + ks * 32), lds32(br + ks * 32 + 16));
      }
#pragma unroll
      for (int e = 0; e < 4; e++) part[(tw * 32 + lane) * 4 + e] = d[e];
    }
    __syncthreads();
    for (int idx = tid; idx < tiles * 32; idx += nt) {
      const int tile = idx >> 5, ln = idx & 31, g8 = ln >> 2, t4 = ln & 3;
      const int m0 = (tile % pm) * 16, n0 = (tile / pm) * 8, h = (n0 >> 1) + t4;
      int32_t d[4] = {0, 0, 0, 0};
      for (int sp = 0; sp < split; sp++)
#pragma unroll
        for (int e = 0; e < 4; e++) d[e] += part[((sp * tiles + tile) * 32 + ln) * 4 + e];
      if (h < G) {
#pragma unroll
        for (int hr = 0; hr < 2; hr++) {  // rows g8 and g8 + 8: (high, low) in d[2hr], d[2hr+1]
          const int i = d0 + m0 + g8 + hr * 8;
          float o = 0.0f;
          if (s_wmax[h] > 0.0f)
            o = __fmul_rn((float)(int)(((uint32_t)d[2 * hr] << 8) + (uint32_t)d[2 * hr + 1]),
                          s_wqs[h]);
          p.out[(size_t)r * p.out_ld + (size_t)(kvh * G + h) * hd + i] = o;
        }
      }
    }
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
  } else {

  // ---- weights w_t = e_t * inv * vs_t: their max per head over the window
  {
    float wl[GM];
#pragma unroll
    for (int h = 0; h < GM; h++) wl[h] = 0.0f;
    for (int j = tid; j < ns; j += nt) {
      if (pos_of(S0 + j) < 0) continue;
      const float vsv = vsm[j];
#pragma unroll
      for (int h = 0; h < GM; h++)
        if (h < G) {
          const float w = __fmul_rn(__fmul_rn(ev[h * cs + j], s_inv[h]), vsv);
          wl[h] = w > wl[h] ? w : wl[h];
        }
    }
#pragma unroll
    for (int h = 0; h < GM; h++) wl[h] = warp_max(wl[h]);
    if (lane == 0)
#pragma unroll
      for (int h = 0; h < GM; h++) s_red[warp][h] = wl[h];
  }
  __syncthreads();
  if (tid < G) {
    float m = s_red[0][tid];
    for (int w = 1; w < nw; w++) m = s_red[w][tid] > m ? s_red[w][tid] : m;
    s_lwmax[tid] = m;
  }
  cluster.sync();
  if (tid < G) {
    float v[8];
#pragma unroll
    for (int c = 0; c < 8; c++) v[c] = c < C ? cluster.map_shared_rank(s_lwmax, c)[tid] : 0.0f;
    float m = 0.0f;
#pragma unroll
    for (int c = 0; c < 8; c++) m = v[c] > m ? v[c] : m;
    s_wmax[tid] = m;
    s_wqs[tid] = __fdiv_rn(m, 65535.0f);
    s_wqi[tid] = m > 0.0f ? __fdiv_rn(65535.0f, m) : 0.0f;
  }
  __syncthreads();

  // ---- P.V over this CTA's slot groups (ops.c:560-625): weights quantised
  // to 16 bits of their max, split in hi / lo bytes; dims x (head, hi / lo)
  // on the tensor cores, 32 slots per step, exact int32 sums
  const int pm = hd >> 4, ptiles = pm * ((2 * G + 7) >> 3);
  int32_t pacc[kTiles][4];
#pragma unroll
  for (int q = 0; q < kTiles; q++) pacc[q][0] = pacc[q][1] = pacc[q][2] = pacc[q][3] = 0;
  for (int ga = 0; ga < ns / 4; ga += vg) {
    const int gb = min(ns / 4, ga + vg), nsl = (gb - ga) * 4, kpad = (nsl + 31) & ~31;
    if (ga) {
      __syncthreads();
      load_v(ga, gb);
    }
    for (int j = tid; j < kpad; j += nt) {
      const int js = ga * 4 + j;
      const bool live = j < nsl && pos_of(S0 + js) >= 0;
#pragma unroll
      for (int h = 0; h < GM; h++)
        if (h < G) {
          int iw = 0;
          if (live && s_wmax[h] > 0.0f) {
            const float x = __fadd_rn(
                __fmul_rn(__fmul_rn(__fmul_rn(ev[h * cs + js], s_inv[h]), vsm[js]), s_wqi[h]),
                0.5f);
            iw = (int)x;
            iw = iw > 65535 ? 65535 : (iw < 0 ? 0 : iw);
          }
          wst[(2 * h) * wld + j] = (uint8_t)(iw >> 8);
          wst[(2 * h + 1) * wld + j] = (uint8_t)(iw & 255);
        }
    }
    cp_async_wait<0>();
    __syncthreads();
#pragma unroll
    for (int q = 0; q < kTiles; q++) {
      const int tile = warp + q * nw;
      if (tile < ptiles) {
        const int m0 = (tile % pm) * 16, n0 = (tile / pm) * 8;
        const int8_t *ar = vst + tig * vld + (m0 + gid) * 4;
        const uint8_t *br = wst + min(n0 + gid, 2 * G - 1) * wld + tig * 4;
        for (int kb = 0; kb < kpad; kb += 32) {
          const int8_t *a = ar + (kb >> 2) * vld;
          mma_s8u8_m16n8k32(pacc[q], lds32(a), lds32(a + 32), lds32(a + 4 * vld),
                            lds32(a + 4 * vld + 32), lds32(br + kb), lds32(br + kb + 16));
        }
      }
    }
  }
  // integer sums meet in the CTA that owns the dimension (dims [d0, d0 + dper))
#pragma unroll
  for (int q = 0; q < kTiles; q++) {
    const int tile = warp + q * nw;
    if (tile < ptiles) {
      const int m0 = (tile % pm) * 16, n0 = (tile / pm) * 8;
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const int i = m0 + gid + (e >> 1) * 8, col = n0 + 2 * tig + (e & 1);
        if (col < 2 * G && pacc[q][e])
          atomicAdd(cluster.map_shared_rank(acc, i / dper) + col * hd + i, pacc[q][e]);
      }
    }
  }
  cluster.sync();
  for (int idx = tid; idx < G * dper; idx += nt) {
    const int h = idx / dper, i = rank * dper + (idx - h * dper);
    float o = 0.0f;
    if (s_wmax[h] > 0.0f)
      o = __fmul_rn((float)(int)(((uint32_t)acc[(2 * h) * hd + i] << 8) +
                                 (uint32_t)acc[(2 * h + 1) * hd + i]),
                    s_wqs[h]);
    p.out[(size_t)r * p.out_ld + (size_t)(kvh * G + h) * hd + i] = o;
  }
  }  // !ONE
}

// ------------------------------------------------------------ fused row ops
// The decode step's glue between GEMMs merged per row so that each merge is
// one launch; every value is computed by the same expressions as the
// separate kernels above, so the results are bit-identical to running them
// one after the other.

// ops.c:59-92: 1 / sqrt(mean of squares + eps) of a row staged in shared
// memory -- 16 lane sums in order, reduced, then the tail.  Called by all
// threads of the CTA.
__device__ float rms_inv(const float *xs, int n, float eps, float *lanes, float *s_val) {
  const int full = n & ~15;
  if (threadIdx.x < 16) {
    lanes[threadIdx.x] = lane_sumsq(xs, threadIdx.x, full);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float ss = reduce16(lanes);
    for (int i = full; i < n; i++) ss = __fmaf_rn(xs[i], xs[i], ss);
    *s_val = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
  }
  __syncthreads();
  return *s_val;
}

// Largest |x| over the CTA's values (each thread passes its own maximum).
__device__ float block_amax(float mx, float *red) {
  mx = warp_max(mx);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = 0.0f;
  for (int w = 0; w < (int)(blockDim.x >> 5); w++) mx = red[w] > mx ? red[w] : mx;
  __syncthreads();  // red may be reused
  return mx;
}

// The prep of a row staged in shared memory with no rotation (ops.c:293-314):
// the symmetric int8 scale of its max (ops.c:181-204), then the row's 64-byte
// pieces of the packed GEMM tiles.  k is a multiple of 64.
// mx: this thread's max |x| over the values it wrote, or -1 to scan the row.
__device__ void quant_pack_row(const float *xs, int k, int r, float *qs, int8_t *pa, float *red,
                               float mx = -1.0f) {
  if (mx < 0.0f) {
    mx = 0.0f;
    __syncthreads();
    for (int i = threadIdx.x; i < k; i += blockDim.x) {
      const float a = fabsf(xs[i]);
      mx = a > mx ? a : mx;
    }
  }
  mx = block_amax(mx, red);  // its first barrier also publishes xs
  const float s = mx == 0.0f ? 1.0f : __fdiv_rn(mx, 127.0f);
  const float inv = __fdiv_rn(1.0f, s);
  if (threadIdx.x == 0) qs[r] = s;
  int8_t *row = pa + (size_t)(r / 16) * (k / kTileK) * kATile + (size_t)(r % 16) * 64;
  for (int i = threadIdx.x * 4; i < k; i += blockDim.x * 4)
    *reinterpret_cast<uint32_t *>(row + (size_t)(i / 64) * kATile + (i % 64)) =
        q8_quad(*reinterpret_cast<const float4 *>(xs + i), inv);
}

// A packed row past the last real row of its 16-row tile: zeros.
__device__ void zero_pack_row(int k, int r, int8_t *pa) {
  int8_t *row = pa + (size_t)(r / 16) * (k / kTileK) * kATile + (size_t)(r % 16) * 64;
  for (int i = threadIdx.x * 4; i < k; i += blockDim.x * 4)
    *reinterpret_cast<uint32_t *>(row + (size_t)(i / 64) * kATile + (i % 64)) = 0u;
}

// forward.rs:625-640 + :476-480: when proj is given, h += rmsnorm(proj, w_post)
// (ops.c:59-92 then ops.c:317-321); then the next GEMM's packed rows of
// rmsnorm(h, w_pre).  One CTA per row, rows [m, 16-row tile end) zero-filled.
// Rows go through shared memory whole (all loads in flight at once), h is
// written back last.
__global__ void __launch_bounds__(kGlueThreads) norm_prep_kernel(
    float *__restrict__ h, const float *__restrict__ proj, const float *__restrict__ w_post,
    const float *__restrict__ w_pre, int m, int n, float eps, float *__restrict__ qs,
    int8_t *__restrict__ pa) {
  // shared memory: [n] the row to normalise, [n] the residual, [n] w_post, [n] w_pre
  extern __shared__ __align__(16) float xs[];
  __shared__ float lanes[16], red[32], s_val;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int r = blockIdx.x, n4 = n >> 2;
  if (r >= m) {
    zero_pack_row(n, r, pa);
    return;
  }
  float *hs = xs + n, *wa = xs + 2 * n, *wb = xs + 3 * n;
  float4 *h4 = reinterpret_cast<float4 *>(h + (size_t)r * n);
  const float4 *src[4] = {h4, proj ? reinterpret_cast<const float4 *>(proj + (size_t)r * n) : nullptr,
                          proj ? reinterpret_cast<const float4 *>(w_post) : nullptr,
                          reinterpret_cast<const float4 *>(w_pre)};
  float4 *dst[4] = {reinterpret_cast<float4 *>(hs), reinterpret_cast<float4 *>(xs),
                    reinterpret_cast<float4 *>(wa), reinterpret_cast<float4 *>(wb)};
  // every load of a batch is issued before any shared store
  for (int base = 0; base < n4; base += 2 * kGlueThreads) {
    float4 v[4][2];
#pragma unroll
    for (int a = 0; a < 4; a++)
#pragma unroll
      for (int k = 0; k < 2; k++) {
        const int i = base + k * kGlueThreads + threadIdx.x;
        if (src[a] && i < n4) v[a][k] = src[a][i];
      }
#pragma unroll
    for (int a = 0; a < 4; a++)
#pragma unroll
      for (int k = 0; k < 2; k++) {
        const int i = base + k * kGlueThreads + threadIdx.x;
        if (src[a] && i < n4) dst[a][i] = v[a][k];
      }
  }
  __syncthreads();
  if (proj) {
    const float inv = rms_inv(xs, n, eps, lanes, &s_val);
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const float t = w_post ? __fmul_rn(__fmul_rn(xs[i], inv), wa[i]) : __fmul_rn(xs[i], inv);
      hs[i] = __fadd_rn(hs[i], t);
    }
    __syncthreads();
  }
  const float inv = rms_inv(hs, n, eps, lanes, &s_val);
  float mx = 0.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float y = w_pre ? __fmul_rn(__fmul_rn(hs[i], inv), wb[i]) : __fmul_rn(hs[i], inv);
    xs[i] = y;
    mx = fabsf(y) > mx ? fabsf(y) : mx;
  }
  if (proj)
    for (int i = threadIdx.x; i < n4; i += blockDim.x) h4[i] = reinterpret_cast<float4 *>(hs)[i];
  quant_pack_row(xs, n, r, qs, pa, red, mx);
}

// ops.c:119-131 then the prep: the down projection's packed rows of
// gelu(gate) * up, gate and up rows ld floats apart (optionally the f32
// product too, rows of n).  A cluster of C CTAs per
// row, each on n / C columns; the row's max meets through distributed
// shared memory.
__global__ void __launch_bounds__(kGlueThreads) gelu_mul_prep_kernel(
    const float *__restrict__ gate, const float *__restrict__ up, int ld, int m, int n,
    float *__restrict__ act, float *__restrict__ qs, int8_t *__restrict__ pa) {
  cg::cluster_group cluster = cg::this_cluster();
  extern __shared__ __align__(16) float xs[];
  __shared__ float red[32], s_amax;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int C = (int)cluster.num_blocks(), rank = (int)cluster.block_rank();
  const int r = blockIdx.y, w = n / C, c0 = rank * w;  // w: a multiple of 64
  int8_t *row = pa + (size_t)(r / 16) * (n / kTileK) * kATile + (size_t)(r % 16) * 64;
  if (r >= m) {  // the whole cluster is a padding row
    for (int i = threadIdx.x * 4; i < w; i += blockDim.x * 4)
      *reinterpret_cast<uint32_t *>(row + (size_t)((c0 + i) / 64) * kATile + ((c0 + i) % 64)) = 0u;
    return;
  }
  const float4 *g4 = reinterpret_cast<const float4 *>(gate + (size_t)r * ld + c0);
  const float4 *u4 = reinterpret_cast<const float4 *>(up + (size_t)r * ld + c0);
  const int full = n & ~15;
  float mx = 0.0f;
#pragma unroll 2
  for (int i = threadIdx.x; i < w / 4; i += blockDim.x) {
    const float4 g = g4[i], u = u4[i];
    const int c = c0 + 4 * i;
    float4 v;
    v.x = __fmul_rn(c < full ? gelu_lane(g.x) : gelu_tail(g.x), u.x);
    v.y = __fmul_rn(c + 1 < full ? gelu_lane(g.y) : gelu_tail(g.y), u.y);
    v.z = __fmul_rn(c + 2 < full ? gelu_lane(g.z) : gelu_tail(g.z), u.z);
    v.w = __fmul_rn(c + 3 < full ? gelu_lane(g.w) : gelu_tail(g.w), u.w);
    reinterpret_cast<float4 *>(xs)[i] = v;
    const float a = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    mx = a > mx ? a : mx;
  }
  mx = block_amax(mx, red);
  if (threadIdx.x == 0) s_amax = mx;
  cluster.sync();
  float v[8];
#pragma unroll
  for (int c = 0; c < 8; c++)
    v[c] = c < C ? *cluster.map_shared_rank(&s_amax, c) : 0.0f;
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");  // done with the peers
  mx = 0.0f;
#pragma unroll
  for (int c = 0; c < 8; c++) mx = v[c] > mx ? v[c] : mx;
  const float s = mx == 0.0f ? 1.0f : __fdiv_rn(mx, 127.0f);
  const float inv = __fdiv_rn(1.0f, s);
  if (rank == 0 && threadIdx.x == 0) qs[r] = s;
  for (int i = threadIdx.x; i < w / 4; i += blockDim.x) {
    const float4 x = reinterpret_cast<const float4 *>(xs)[i];
    const int c = c0 + 4 * i;
    *reinterpret_cast<uint32_t *>(row + (size_t)(c / 64) * kATile + (c % 64)) = q8_quad(x, inv);
    if (act) *reinterpret_cast<float4 *>(act + (size_t)r * n + c) = x;
  }
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// forward.rs:482-545 for one row: rmsnorm of each query head (q_norm) and
// key head (k_norm) then rope (ops.c:135-147), each value head without
// scale; then the key and value rows quantised to int8 with one scale each
// (ops.c:181-204) into the row's caches at slot pos (mod ring): K as a row
// of the [slot][kv_heads * head_dim] cache, V into the slot-interleaved
// layout (ops.c:653-660).  q, k and v keep the normalised (and rotated)
// values, like the reference's buffers.  A slot outside [0, cap) writes no
// cache entry.
__global__ void __launch_bounds__(kGlueThreads) qkv_post_kernel(const QkvParams p) {
  // shared memory: q heads, k heads, v heads; then cos, sin [hd / 2] each, q_norm, k_norm
  extern __shared__ __align__(16) float xs[];
  __shared__ float lanes[48][16], inv_h[48], red[32];
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int r = blockIdx.x, hd = p.head_dim, half = hd / 2;
  const int nq = p.n_heads * hd, kvd = p.kv_heads * hd, heads = p.n_heads + 2 * p.kv_heads;
  float *qr = p.q + (size_t)r * p.q_ld, *kr = p.k + (size_t)r * p.kv_ld,
        *vr = p.v + (size_t)r * p.kv_ld;
  float *cs = xs + nq + 2 * kvd, *sn = cs + half, *qn = sn + half, *kn = qn + hd;
  const int pos = p.pos[r];
  {  // q, k and v rows as float4, every load of a batch before any shared store
    const int q4 = nq >> 2, k4 = kvd >> 2, tot = q4 + 2 * k4;
    float4 *x4 = reinterpret_cast<float4 *>(xs);
    for (int base = 0; base < tot; base += 4 * kGlueThreads) {
      float4 v[4];
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const int i = base + k * kGlueThreads + threadIdx.x;
        if (i < tot)
          v[k] = i < q4 ? reinterpret_cast<const float4 *>(qr)[i]
                        : (i < q4 + k4 ? reinterpret_cast<const float4 *>(kr)[i - q4]
                                       : reinterpret_cast<const float4 *>(vr)[i - q4 - k4]);
      }
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const int i = base + k * kGlueThreads + threadIdx.x;
        if (i < tot) x4[i] = v[k];
      }
    }
  }
  for (int j = threadIdx.x; j < hd; j += blockDim.x) {
    const float wq = p.q_norm[j], wk = p.k_norm[j];
    qn[j] = wq;
    kn[j] = wk;
    if (j < half) rope_cs(p.inv_freq, p.rope_tab, p.rope_positions, half, pos, j, cs[j], sn[j]);
  }
  __syncthreads();
  // per-head sums of squares: a half-warp per head, 16 lanes in order
  for (int hh = threadIdx.x >> 4; hh < heads; hh += blockDim.x >> 4) {
    const float *x = xs + hh * hd;
    lanes[hh][threadIdx.x & 15] = lane_sumsq(x, threadIdx.x & 15, hd & ~15);
  }
  __syncthreads();
  if (threadIdx.x < heads) {  // ops.c:59-92: reduced lanes, then the tail past the last 16
    const float *x = xs + threadIdx.x * hd;
    float ss = reduce16(lanes[threadIdx.x]);
    for (int i = hd & ~15; i < hd; i++) ss = __fmaf_rn(x[i], x[i], ss);
    inv_h[threadIdx.x] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)hd), p.eps)));
  }
  __syncthreads();
  // a warp per head: the norm, rope on query and key heads (pairs j, j +
  // half), the result stored to the row and, for k and v, kept for the cache
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  float kmx = 0.0f, vmx = 0.0f;
  for (int hh = warp; hh < heads; hh += nw) {
    float *x = xs + hh * hd;
    const float inv = inv_h[hh];
    const bool is_q = hh < p.n_heads, is_v = hh >= p.n_heads + p.kv_heads;
    const float *w = is_q ? qn : kn;
    float *dst = is_q ? qr + (size_t)hh * hd
                      : (is_v ? vr + (size_t)(hh - p.n_heads - p.kv_heads) * hd
                              : kr + (size_t)(hh - p.n_heads) * hd);
    if (is_v) {
      for (int d = lane; d < hd; d += 32) {
        const float y = __fmul_rn(x[d], inv);
        x[d] = y;
        dst[d] = y;
        vmx = fabsf(y) > vmx ? fabsf(y) : vmx;
      }
    } else {
      for (int j = lane; j < half; j += 32) {
        const float lo = __fmul_rn(__fmul_rn(x[j], inv), w[j]);
        const float hi = __fmul_rn(__fmul_rn(x[j + half], inv), w[j + half]);
        const float rl = __fmaf_rn(lo, cs[j], -__fmul_rn(hi, sn[j]));
        const float rh = __fmaf_rn(hi, cs[j], __fmul_rn(lo, sn[j]));
        x[j] = rl;
        x[j + half] = rh;
        dst[j] = rl;
        dst[j + half] = rh;
        if (!is_q) kmx = fmaxf(kmx, fmaxf(fabsf(rl), fabsf(rh)));
      }
    }
  }
  // int8 K and V rows with one scale each (ops.c:181-204), into the caches
  const int slot = p.ring ? pos % p.ring : pos;
  if (slot < 0 || slot >= p.cap) return;  // no cache entry for this row (whole CTA)
  kmx = warp_max(kmx);
  vmx = warp_max(vmx);
  if (lane == 0) {
    red[warp] = kmx;
    red[16 + warp] = vmx;
  }
  __syncthreads();
  kmx = vmx = 0.0f;
  for (int w = 0; w < nw; w++) {
    kmx = red[w] > kmx ? red[w] : kmx;
    vmx = red[16 + w] > vmx ? red[16 + w] : vmx;
  }
  const float ksc = kmx == 0.0f ? 1.0f : __fdiv_rn(kmx, 127.0f);
  const float vsc = vmx == 0.0f ? 1.0f : __fdiv_rn(vmx, 127.0f);
  const float kinv = __fdiv_rn(1.0f, ksc), vinv = __fdiv_rn(1.0f, vsc);
  const float *xk = xs + nq, *xv = xs + nq + kvd;
  int8_t *kd = p.kc + (size_t)r * p.kc_stride + (size_t)slot * kvd;
  int8_t *vd = p.vt + (size_t)r * p.vt_stride + (size_t)(slot >> 2) * kvd * 4 + (slot & 3);
  for (int i = threadIdx.x; i < kvd; i += blockDim.x) {
    kd[i] = (int8_t)q8_x86(__fmul_rn(xk[i], kinv));
    vd[(size_t)i * 4] = (int8_t)q8_x86(__fmul_rn(xv[i], vinv));
  }
  if (threadIdx.x == 0) {
    p.ks[(size_t)r * p.ks_stride + slot] = ksc;
    p.vs[(size_t)r * p.vs_stride + slot] = vsc;
  }
}

template <class K, class... A>
cudaError_t launch_pdl(K kern, dim3 grid, dim3 block, size_t smem, bool pdl, cudaStream_t st,
                       A... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

unsigned grid_for(size_t n) {
  size_t b = (n + kGlueThreads - 1) / kGlueThreads;
  return (unsigned)(b > 1184 ? 1184 : (b ? b : 1));
}

}  // namespace

cudaError_t launch_norm_prep(float *h, const float *proj, const float *w_post, const float *w_pre,
                             int m, int n, float eps, float *qs, int8_t *pa, bool pdl,
                             cudaStream_t st) {
  const size_t smem = (size_t)n * 16;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(norm_prep_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  return launch_pdl(norm_prep_kernel, dim3((unsigned)((m + 15) & ~15)), dim3(kGlueThreads), smem,
                    pdl, st, h, proj, w_post, w_pre, m, n, eps, qs, pa);
}

cudaError_t launch_gelu_mul_prep(const float *gate, const float *up, int ld, int m, int n,
                                 float *act, float *qs, int8_t *pa, bool pdl, cudaStream_t st) {
  int c = 8;
  while ((n / 64) % c) c >>= 1;  // whole 64-column tiles per CTA
  const size_t smem = (size_t)(n / c) * 4;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(gelu_mul_prep_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)c, (unsigned)((m + 15) & ~15));
  cfg.blockDim = dim3(kGlueThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)c;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, gelu_mul_prep_kernel, gate, up, ld, m, n, act, qs, pa);
}

size_t qkv_post_smem(const QkvParams &p) {
  return ((size_t)(p.n_heads + 2 * p.kv_heads) * p.head_dim + 3 * (size_t)p.head_dim) * 4;
}

cudaError_t launch_qkv_post(const QkvParams &p, int rows, bool pdl, cudaStream_t st) {
  const size_t smem = qkv_post_smem(p);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(qkv_post_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  return launch_pdl(qkv_post_kernel, dim3((unsigned)rows), dim3(kGlueThreads), smem, pdl, st, p);
}


cudaError_t launch_rmsnorm(float *out, const float *x, const float *w, int rows, int n, float eps,
                           bool pdl, cudaStream_t st) {
  const size_t smem = (size_t)n * 4;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(rmsnorm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
  }
  return launch_pdl(rmsnorm_kernel, dim3(rows), dim3(kGlueThreads), smem, pdl, st, out, x, w, n,
                    eps);
}

cudaError_t launch_gelu_mul(float *out, const float *gate, const float *up, int rows, int n,
                            bool pdl, cudaStream_t st) {
  const size_t total = (size_t)rows * n;
  return launch_pdl(gelu_mul_kernel, dim3(grid_for(total)), dim3(kGlueThreads), 0, pdl, st, out,
                    gate, up, n, total);
}

cudaError_t launch_elementwise(float *a, const float *b, float s, size_t n, int op, bool pdl,
                               cudaStream_t st) {
  return launch_pdl(elementwise_kernel, dim3(grid_for(n)), dim3(kGlueThreads), 0, pdl, st, a, b, s,
                    n, op);
}

cudaError_t launch_softcap(float *x, int rows, int n, float cap, bool pdl, cudaStream_t st) {
  const size_t total = (size_t)rows * n;
  return launch_pdl(softcap_kernel, dim3(grid_for(total)), dim3(kGlueThreads), 0, pdl, st, x, n,
                    total, cap);
}

cudaError_t launch_rope(float *x, int x_ld, int rows, int n_heads, int head_dim,
                        const float *inv_freq, const float *tab, int positions, const int *pos,
                        bool pdl, cudaStream_t st) {
  const int pairs = n_heads * (head_dim / 2);
  const unsigned gx = (unsigned)((pairs + kGlueThreads - 1) / kGlueThreads);
  return launch_pdl(rope_kernel, dim3(gx, rows), dim3(kGlueThreads), 0, pdl, st, x, x_ld, n_heads,
                    head_dim, inv_freq, tab, positions, pos);
}

cudaError_t launch_store_v_t(int8_t *vt, size_t vt_stride, const int8_t *src, int src_ld, int rows,
                             int n, int slot, bool pdl, cudaStream_t st) {
  const unsigned gx = (unsigned)((n + kGlueThreads - 1) / kGlueThreads);
  return launch_pdl(store_v_t_kernel, dim3(gx, rows), dim3(kGlueThreads), 0, pdl, st, vt,
                    vt_stride, src, src_ld, n, slot);
}

namespace {

unsigned align16(size_t x) { return (unsigned)((x + 15) & ~(size_t)15); }

int gm_of(const AttnParams &p) {
  const int g = p.n_heads / p.kv_heads;
  int gm = 1;
  while (gm < g) gm <<= 1;
  return gm;
}

template <int GM, bool ONE>
cudaError_t launch_attend_gm(const AttnParams &p, int rows, bool pdl, cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(attend_q8_kernel<GM, ONE>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(p.cluster * p.kv_heads), (unsigned)rows);
  cfg.blockDim = dim3(kGlueThreads);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)p.cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, attend_q8_kernel<GM, ONE>, p);
}

}  // namespace

bool attend_layout(AttnParams &p, size_t smem_limit) {
  const int n = p.end - p.start, hd = p.head_dim, gm = gm_of(p);
  if (gm > 16) return false;
  int c = 1;
  while (c < 8 && n >= 64 * c) c <<= 1;  // about 32 positions or more per CTA
  p.cluster = c;
  p.gchunk = (p.wslots / 4 + c - 1) / c;
  const int cs = 4 * p.gchunk;
  const int win_max = (4096 / gm) & ~15;
  p.win = win_max < ((n + 15) & ~15) ? win_max : ((n + 15) & ~15);
  const size_t kld = (size_t)hd + 16, vld = (size_t)hd * 4 + 32;
  const size_t base = align16((size_t)gm * hd) + align16((size_t)2 * cs * 4) +
                      align16((size_t)gm * cs * 4) + align16((size_t)gm * p.win * 4) +
                      4096;  // + static shared memory
  // single-window form: all V groups of this CTA's dims, all weight bytes,
  // all V scales, the P.V partial sums in the K stage
  p.one = ((n + 15) & ~15) <= win_max && (hd / c) % 16 == 0;
  if (p.one) {
    const int kpad = (p.wslots + 31) & ~31;
    const int tiles = (hd / c / 16) * ((2 * (p.n_heads / p.kv_heads) + 7) / 8);
    const size_t part = (size_t)(tiles > 8 ? tiles : 8) * 512;
    p.kp = cs < kGlueThreads ? ((cs + 15) & ~15) : kGlueThreads;
    size_t kbytes = align16((size_t)p.kp * kld);
    if (kbytes < part) kbytes = align16(part);
    if (kbytes < (size_t)gm * kpad * 4) kbytes = align16((size_t)gm * kpad * 4);  // weights
    p.vg = p.gchunk;
    p.vgp = kpad / 4;
    p.off_ks = align16((size_t)gm * hd);
    p.off_k = p.off_ks + align16((size_t)2 * cs * 4);
    p.off_v = p.off_k + (unsigned)kbytes;
    p.off_e = p.off_v + align16((size_t)p.vgp * ((size_t)hd / c * 4 + 32));
    p.off_win = p.off_e + align16((size_t)gm * cs * 4);
    p.off_w = p.off_win + align16((size_t)gm * p.win * 4);
    p.off_vsa = p.off_w + align16((size_t)2 * gm * (p.vgp * 4 + 16));
    p.off_acc = p.off_vsa + align16((size_t)p.wslots * 4);
    p.smem = p.off_acc;
    if (p.smem + 4096 <= smem_limit) return true;
    p.one = 0;
  }
  const size_t fixed = base + (size_t)gm * 2 * hd * 4;
  // smallest stages: 16 K rows, 8 V groups with their weight bytes
  const size_t kv_min = 16 * kld + 8 * vld + 2 * (size_t)gm * (32 + 16);
  if (fixed + kv_min > smem_limit) return false;
  const size_t stage = (smem_limit - fixed) / 2 < 65536 ? (smem_limit - fixed) / 2 : 65536;
  p.kp = (int)(stage / kld) & ~15;
  if (p.kp > ((cs + 15) & ~15)) p.kp = (cs + 15) & ~15;
  if (p.kp > kGlueThreads) p.kp = kGlueThreads;
  if (p.kp < 16) p.kp = 16;
  p.vg = (int)(stage / (vld + 2 * (size_t)gm * 4)) & ~7;
  if (p.vg > p.gchunk) p.vg = p.gchunk;
  if (p.vg < 1) p.vg = 1;
  p.vgp = (p.vg + 7) & ~7;
  p.off_ks = align16((size_t)gm * hd);
  p.off_k = p.off_ks + align16((size_t)2 * cs * 4);
  p.off_v = p.off_k + align16((size_t)p.kp * kld);
  p.off_e = p.off_v + align16((size_t)p.vgp * vld);
  p.off_win = p.off_e + align16((size_t)gm * cs * 4);
  p.off_w = p.off_win + align16((size_t)gm * p.win * 4);
  p.off_vsa = p.off_w + align16((size_t)2 * gm * (p.vgp * 4 + 16));
  p.off_acc = p.off_vsa;
  p.smem = p.off_acc + (size_t)gm * 2 * hd * 4;
  return p.smem + 4096 <= smem_limit;
}

cudaError_t launch_attend_q8(const AttnParams &p, int rows, bool pdl, size_t smem_limit,
                             cudaStream_t st) {
  if (p.smem + 4096 > smem_limit) return cudaErrorInvalidConfiguration;
  switch (gm_of(p) * 2 + (p.one ? 1 : 0)) {
    case 2: return launch_attend_gm<1, false>(p, rows, pdl, st);
    case 3: return launch_attend_gm<1, true>(p, rows, pdl, st);
    case 4: return launch_attend_gm<2, false>(p, rows, pdl, st);
    case 5: return launch_attend_gm<2, true>(p, rows, pdl, st);
    case 8: return launch_attend_gm<4, false>(p, rows, pdl, st);
    case 9: return launch_attend_gm<4, true>(p, rows, pdl, st);
    case 16: return launch_attend_gm<8, false>(p, rows, pdl, st);
    case 17: return launch_attend_gm<8, true>(p, rows, pdl, st);
    case 32: return launch_attend_gm<16, false>(p, rows, pdl, st);
    case 33: return launch_attend_gm<16, true>(p, rows, pdl, st);
    default: return cudaErrorInvalidConfiguration;
  }
}

}  // namespace fgm
