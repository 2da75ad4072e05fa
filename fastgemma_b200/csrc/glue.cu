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
// Attention (ops.c:378-640) is one CTA per (query row, head): the per-head
// int8 quantisation of Q, exact int8 Q.K dot products (dp4a), the softmax
// with the reference's lane order for the sum, the 16-bit split weights and
// the exact P.V against the slot-interleaved V cache (dp4a, unsigned weight
// bytes times signed V bytes).  Integer sums are exact in any order; every
// float step follows the reference's order, so the output is bit-identical.

#include "fgm_common.cuh"
#include "fgm_internal.h"

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
    float acc = 0.0f;
    for (int i = threadIdx.x; i < full; i += 16) acc = __fmaf_rn(xs[i], xs[i], acc);
    lanes[threadIdx.x] = acc;
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

// ops.c:135-147 for `rows` rows (row r at x + r*x_ld, position pos[r]).  The
// reference's build fuses each product pair into one rounding.
__global__ void rope_kernel(float *x, int x_ld, int n_heads, int head_dim, const float *inv_freq,
                            const int *pos) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int h = head_dim / 2, r = blockIdx.y;
  float *xr = x + (size_t)r * x_ld;
  for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < n_heads * h;
       idx += gridDim.x * blockDim.x) {
    const int hh = idx / h, j = idx % h;
    const float a = __fmul_rn((float)pos[r], inv_freq[j]);
    const float c = (float)cos((double)a), s = (float)sin((double)a);
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

__device__ __forceinline__ int dp4a_ss(int a, int b, int c) {
  int d;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// signed V bytes times unsigned weight bytes
__device__ __forceinline__ int dp4a_su(int a, unsigned b, int c) {
  int d;
  asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ float block_max(float v, float *red) {
  for (int o = 16; o > 0; o >>= 1) {
    const float u = __shfl_xor_sync(0xffffffffu, v, o);
    v = u > v ? u : v;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float m = red[0];
  for (int w = 1; w < (int)(blockDim.x >> 5); w++) m = red[w] > m ? red[w] : m;
  return m;
}

// ops.c:378-640, one (head, query row) per CTA.  Shared memory: the row's
// scores [n], the slot-indexed weight bytes hi / lo [W] (W: cache slots that
// can be touched, a multiple of 4), Q as int8.
__global__ void __launch_bounds__(kGlueThreads) attend_q8_kernel(const AttnParams p) {
  extern __shared__ __align__(16) uint8_t sm[];
  __shared__ float red[32];
  __shared__ float lanes[16];
  __shared__ float s_sum;
  __shared__ __align__(16) int8_t qq[512];
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int h = blockIdx.x, r = blockIdx.y;
  const int hd = p.head_dim, kvd = p.kv_heads * hd, kvh = h / (p.n_heads / p.kv_heads);
  const int n = p.end - p.start, W = p.wslots;
  float *sc = reinterpret_cast<float *>(sm);
  uint8_t *whi = sm + (size_t)n * 4, *wlo = whi + W;
  const float *qh = p.q + (size_t)r * p.q_ld + (size_t)h * hd;
  const int8_t *kc = p.kc + (size_t)r * p.kc_stride;
  const float *ks = p.ks + (size_t)r * p.ks_stride;
  const int8_t *vt = p.vt + (size_t)r * p.vt_stride;
  const float *vs = p.vs + (size_t)r * p.vs_stride;
  float *oh = p.out + (size_t)r * p.out_ld + (size_t)h * hd;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;

  // ---- Q per head: int8 with one scale (ops.c:412-431)
  float a = 0.0f;
  for (int i = tid; i < hd; i += blockDim.x) {
    const float v = fabsf(qh[i]);
    a = v > a ? v : a;
  }
  const float qamax = block_max(a, red);
  const float qscale = __fdiv_rn(qamax, 127.0f);
  const float qinv = qamax > 0.0f ? __fdiv_rn(127.0f, qamax) : 0.0f;
  for (int i = tid; i < hd; i += blockDim.x) {
    int v = __float2int_rn(__fmul_rn(qh[i], qinv));
    qq[i] = (int8_t)(v > 127 ? 127 : (v < -127 ? -127 : v));
  }
  for (int i = tid; i < W; i += blockDim.x) whi[i] = wlo[i] = 0;
  __syncthreads();

  // ---- scores: one warp per position, exact int8 dot (ops.c:432-474)
  const int words = hd / 4;
  const int *q4 = reinterpret_cast<const int *>(qq);
  float mloc = -INFINITY;
  for (int t = p.start + warp; t < p.end; t += nw) {
    const int sl = p.ring ? t % p.ring : t;
    const int *kp = reinterpret_cast<const int *>(kc + (size_t)sl * kvd + (size_t)kvh * hd);
    int dot = 0;
    for (int wi = lane; wi < words; wi += 32) dot = dp4a_ss(kp[wi], q4[wi], dot);
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    const float s = __fmul_rn(__fmul_rn((float)dot, qscale), ks[sl]);
    if (lane == 0) sc[t - p.start] = s;
    mloc = s > mloc ? s : mloc;
  }
  const float mx = block_max(mloc, red);

  // ---- softmax: exp lanes over the 16-position chunks, libm on the tail;
  // the sum in the reference's order (per lane, reduced, then the tail)
  const int full = n & ~15;
  for (int u = tid; u < n; u += blockDim.x) {
    const float d = __fsub_rn(sc[u], mx);
    sc[u] = u < full ? exp_lane(d) : (float)exp((double)d);
  }
  __syncthreads();
  if (tid < 16) {
    float l = 0.0f;
    for (int u = tid; u < full; u += 16) l = __fadd_rn(l, sc[u]);
    lanes[tid] = l;
  }
  __syncthreads();
  if (tid == 0) {
    float sum = reduce16(lanes);
    for (int u = full; u < n; u++) sum = __fadd_rn(sum, sc[u]);
    s_sum = sum;
  }
  __syncthreads();
  const float inv = __fdiv_rn(1.0f, s_sum);

  // ---- weights w_t = e_t * inv * vs_t, quantised to 16 bits of their max
  float wl = 0.0f;
  for (int t = p.start + tid; t < p.end; t += blockDim.x) {
    const float w = __fmul_rn(__fmul_rn(sc[t - p.start], inv), vs[p.ring ? t % p.ring : t]);
    wl = w > wl ? w : wl;
  }
  const float wmax = block_max(wl, red);
  if (!(wmax > 0.0f)) {
    for (int i = tid; i < hd; i += blockDim.x) oh[i] = 0.0f;
    return;
  }
  const float wq_scale = __fdiv_rn(wmax, 65535.0f), wq_inv = __fdiv_rn(65535.0f, wmax);
  for (int t = p.start + tid; t < p.end; t += blockDim.x) {
    const int sl = p.ring ? t % p.ring : t;
    const float x = __fadd_rn(
        __fmul_rn(__fmul_rn(__fmul_rn(sc[t - p.start], inv), vs[sl]), wq_inv), 0.5f);
    int iw = (int)x;
    iw = iw > 65535 ? 65535 : (iw < 0 ? 0 : iw);
    whi[sl - p.wbase] = (uint8_t)(iw >> 8);
    wlo[sl - p.wbase] = (uint8_t)(iw & 255);
  }
  __syncthreads();

  // ---- P.V against the slot-interleaved V cache (ops.c:560-625): thread
  // per dim, four slots per dp4a, exact int32 sums
  const uint32_t *wh4 = reinterpret_cast<const uint32_t *>(whi);
  const uint32_t *wl4 = reinterpret_cast<const uint32_t *>(wlo);
  for (int i = tid; i < hd; i += blockDim.x) {
    int ah = 0, al = 0;
    for (int g = 0; g < W / 4; g++) {
      const uint32_t bh = wh4[g], bl = wl4[g];
      if ((bh | bl) == 0) continue;
      const int v = *reinterpret_cast<const int *>(
          vt + (((size_t)(p.wbase / 4 + g) * kvd + (size_t)kvh * hd + i) * 4));
      ah = dp4a_su(v, bh, ah);
      al = dp4a_su(v, bl, al);
    }
    oh[i] = __fmul_rn((float)(int)(((uint32_t)ah << 8) + (uint32_t)al), wq_scale);
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
                        const float *inv_freq, const int *pos, bool pdl, cudaStream_t st) {
  const int pairs = n_heads * (head_dim / 2);
  const unsigned gx = (unsigned)((pairs + kGlueThreads - 1) / kGlueThreads);
  return launch_pdl(rope_kernel, dim3(gx, rows), dim3(kGlueThreads), 0, pdl, st, x, x_ld, n_heads,
                    head_dim, inv_freq, pos);
}

cudaError_t launch_store_v_t(int8_t *vt, size_t vt_stride, const int8_t *src, int src_ld, int rows,
                             int n, int slot, bool pdl, cudaStream_t st) {
  const unsigned gx = (unsigned)((n + kGlueThreads - 1) / kGlueThreads);
  return launch_pdl(store_v_t_kernel, dim3(gx, rows), dim3(kGlueThreads), 0, pdl, st, vt,
                    vt_stride, src, src_ld, n, slot);
}

size_t attend_smem_bytes(const AttnParams &p) {
  return (size_t)(p.end - p.start) * 4 + 2 * (size_t)p.wslots;
}

cudaError_t launch_attend_q8(const AttnParams &p, int rows, bool pdl, size_t smem_limit,
                             cudaStream_t st) {
  const size_t smem = attend_smem_bytes(p);
  if (smem + 2048 > smem_limit) return cudaErrorInvalidConfiguration;
  cudaError_t e = cudaFuncSetAttribute(attend_q8_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(attend_q8_kernel, dim3(p.n_heads, rows), dim3(kGlueThreads), smem, pdl, st, p);
}

}  // namespace fgm
