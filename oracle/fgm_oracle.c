/*
 * fgm_oracle.c -- CPU restatement of fastgemma's quantised-GEMM hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker the CUDA kernels are
 * compared against.  Nothing in the shipped library links, loads or calls it:
 * only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg do.
 *
 * Every routine is scalar C written from the arithmetic the reference
 * specifies, with the reference file:line it follows.  Paths are relative to
 * the fastgemma project root.
 *
 * Parity pin: the outputs of this file are checked bit-for-bit against
 *   (a) the reference kernels themselves (crates/fgm-kernels/csrc/*.c, compiled
 *       from their own sources into oracle/_ref/ by oracle/Makefile), live, and
 *   (b) golden vectors produced from those reference kernels and committed
 *       under tests/golden/ (see tests/golden/make_golden.py).
 *
 * Arithmetic conventions that make bit-exact parity possible:
 *  - int4 nibbles are two's complement: v -> (v ^ 8) - 8
 *    (amx_gemm.c:84-86, vnni_gemm.c:98-113, vnni_test.c:53-69).
 *  - q4g epilogue: C = 0; for each K group g in ascending order
 *    C = fmaf((float)acc_g, (float)scale_f16[g][n], C); then C *= a_scale[m]
 *    (amx_gemm.c:103-113 drain16 + :365-371; vnni_gemm.c:272-287 + :316-321).
 *  - q8c epilogue: C = (float)acc * (b_scale[n] * a_scale[m])
 *    (amx_gemm.c:399, :433; vnni_gemm.c:207-217).
 *  - activation quantisation: round-to-nearest-even with x86 cvtps_epi32
 *    semantics, then signed saturation to int8 (ops.c:181-204).
 *
 * Build: gcc -O2 -fPIC -shared -ffp-contract=off (oracle/Makefile).  FP
 * contraction must stay off so that only the explicit fmaf() calls fuse.
 */
#include <stdint.h>
#include <stddef.h>
#include <string.h>
#include <math.h>

#define TILE_ROWS 16   /* packed-A rows per tile (ops.c:279-290) */
#define TILE_K 64      /* K values per tile */
#define Q4_TILE 512    /* packed int4 tile bytes (amx_gemm.c:249) */
#define Q8_TILE 1024   /* int8 tile bytes (amx_gemm.c:250) */

/* IEEE binary16 -> binary32, exact for every half value (F16C vcvtph2ps /
 * _cvtsh_ss semantics as used at vnni_gemm.c:283-286 and vnni_test.c:113). */
float orc_f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h >> 15) << 31;
  uint32_t e = (h >> 10) & 0x1f, man = h & 0x3ff, bits;
  if (e == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal: renormalise */
      int shifts = 0;
      while (!(man & 0x400)) { man <<= 1; shifts++; }
      bits = sign | ((uint32_t)(113 - shifts) << 23) | ((man & 0x3ff) << 13);
    }
  } else if (e == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((e + 112) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

/* Two's-complement 4-bit sign extension (vnni_test.c:53, amx_gemm.c:84-86). */
int orc_nibble(int v) { return ((v & 0xF) ^ 8) - 8; }

/* Element (m, k) of a tile-packed activation [ceil(M/16)][K/64][16][64]
 * (ops.c:279-290). */
static inline int a_at(const int8_t *Ap, int KB, int m, int k) {
  return Ap[((size_t)(m / TILE_ROWS) * KB + k / TILE_K) * 1024 +
            (size_t)(m % TILE_ROWS) * 64 + k % TILE_K];
}

/* W[n][k] of an int8 tile blob [N/16][K/64][k/4][n%16][k%4]
 * (convert/quant.py:96-107 pack_b_tiles; vnni_test.c:50 bpos). */
static inline int w8_at(const int8_t *B, int KB, int n, int k) {
  return B[((size_t)(n / 16) * KB + k / TILE_K) * Q8_TILE +
           (size_t)((k % 64) / 4) * 64 + (n % 16) * 4 + k % 4];
}

/* W[n][k] of an int4 tile blob: the int8 tile order above, then cut into
 * 64-value rows whose value i (< 32) is the low nibble of byte i and value
 * i + 32 the high nibble of byte i (convert/quant.py:76-82 pack_nibbles;
 * amx_gemm.c:80-89 unpack64; vnni_test.c:101-109). */
static inline int w4_at(const uint8_t *Bq, int KB, int n, int k) {
  int i = (n % 16) * 4 + k % 4; /* value index inside the 64-value row */
  const uint8_t *row = Bq + ((size_t)(n / 16) * KB + k / TILE_K) * Q4_TILE +
                       (size_t)((k % 64) / 4) * 32;
  int byte = row[i % 32];
  return orc_nibble(i < 32 ? (byte & 0xF) : (byte >> 4));
}

/* ------------------------------------------------------------------ prep */

/* Normalised fast Walsh-Hadamard transform on contiguous hsz-blocks, in the
 * reference's stage order (ops.c:153-175): for len = 1, 2, 4, ... every pair
 * (j, j + len) becomes (u + v, u - v); then each element is multiplied by
 * 1/sqrtf(hsz).  The reference scales in 16-wide chunks only
 * (`i + 16 <= hsz`, ops.c:172), so blocks smaller than 16 stay unscaled; that
 * is reproduced here. */
void orc_fwht(float *x, int n, int hsz) {
  const float scale = 1.0f / sqrtf((float)hsz);
  for (int b = 0; b < n; b += hsz) {
    float *p = x + b;
    for (int len = 1; len < hsz; len <<= 1)
      for (int i = 0; i < hsz; i += len << 1)
        for (int j = i; j < i + len; j++) {
          float u = p[j], v = p[j + len];
          p[j] = u + v;
          p[j + len] = u - v;
        }
    const int scaled = hsz / 16 * 16; /* the 16-wide chunks ops.c:172 covers */
    for (int i = 0; i < scaled; i++) p[i] = p[i] * scale;
  }
}

/* _mm512_cvtps_epi32 (round to nearest even; NaN or |v| >= 2^31 gives
 * INT32_MIN) followed by _mm512_cvtsepi32_epi8 (signed saturation), the
 * conversion pair at ops.c:195-196. */
int8_t orc_cvt_sat_i8(float v) {
  int32_t i;
  if (!(v >= -2147483648.0f && v < 2147483648.0f)) i = INT32_MIN;
  else i = (int32_t)nearbyintf(v); /* default rounding mode: nearest even */
  if (i > 127) i = 127;
  if (i < -128) i = -128;
  return (int8_t)i;
}

/* Per-row symmetric int8 quantisation (ops.c:181-204):
 *   m = max|x|; s = m == 0 ? 1 : m / 127; inv = 1 / s; q = sat8(rne(x * inv)).
 * Rows containing NaN are outside the contract (the reference's vector max
 * keeps or drops a NaN depending on its lane position). */
void orc_quant_act(const float *x, int rows, int k, int8_t *q, float *scale) {
  for (int r = 0; r < rows; r++) {
    const float *src = x + (size_t)r * k;
    float m = 0.0f;
    for (int i = 0; i < k; i++) {
      float a = fabsf(src[i]);
      if (a > m) m = a;
    }
    float s = (m == 0.0f) ? 1.0f : m / 127.0f;
    float inv = 1.0f / s;
    scale[r] = s;
    for (int i = 0; i < k; i++) q[(size_t)r * k + i] = orc_cvt_sat_i8(src[i] * inv);
  }
}

/* Tile-pack a row-major int8 [M, K] into [ceil(M/16)][K/64][16][64], padding
 * rows zero (ops.c:279-290). */
void orc_pack_a(int M, int K, const int8_t *A, int8_t *Ap) {
  const int KB = K / 64, MB = (M + 15) / 16;
  for (int mb = 0; mb < MB; mb++)
    for (int kb = 0; kb < KB; kb++) {
      int8_t *d = Ap + ((size_t)mb * KB + kb) * 1024;
      for (int r = 0; r < 16; r++) {
        int m = mb * 16 + r;
        if (m < M) memcpy(d + r * 64, A + (size_t)m * K + kb * 64, 64);
        else memset(d + r * 64, 0, 64);
      }
    }
}

/* Rows [r0, r1) of the GEMM activation preamble: copy -> FWHT -> quantise ->
 * pack (ops.c:293-314).  r0 must be a multiple of 16. */
void orc_prep_rows(const float *src, int lda, float *rot, int8_t *qa, float *qs,
                   int8_t *pa, int m, int k, int hsz, int r0, int r1) {
  if (r0 >= r1) return;
  const int n = r1 - r0;
  for (int r = r0; r < r1; r++)
    memcpy(rot + (size_t)r * k, src + (size_t)r * lda, (size_t)k * sizeof(float));
  if (hsz > 0) orc_fwht(rot + (size_t)r0 * k, n * k, hsz);
  orc_quant_act(rot + (size_t)r0 * k, n, k, qa + (size_t)r0 * k, qs + r0);
  const int KB = k / 64;
  for (int mb = r0 / 16; mb * 16 < r1; mb++)
    for (int kb = 0; kb < KB; kb++) {
      int8_t *d = pa + ((size_t)mb * KB + kb) * 1024;
      for (int rr = 0; rr < 16; rr++) {
        int row = mb * 16 + rr;
        if (row < m) memcpy(d + rr * 64, qa + (size_t)row * k + kb * 64, 64);
        else memset(d + rr * 64, 0, 64);
      }
    }
}

/* ------------------------------------------------------------------ GEMMs */

/* int32 group accumulators of the int4 GEMM:
 *   acc[m][g][n] = sum_{k in group g} A[m][k] * W[n][k]
 * for n in [n0*16, n1*16).  Output layout [M][K/group][N].  Summed in int64
 * and narrowed: the reference's int32 lanes never wrap for any K the format
 * admits (|sum| <= K * 127 * 8). */
void orc_gemm_q4g_acc(int M, int N, int K, const int8_t *Ap, const uint8_t *Bq,
                      int group, int32_t *acc, int n0, int n1) {
  const int KB = K / 64, G = K / group;
  for (int m = 0; m < M; m++)
    for (int g = 0; g < G; g++)
      for (int n = n0 * 16; n < n1 * 16; n++) {
        int64_t s = 0;
        for (int k = g * group; k < (g + 1) * group; k++)
          s += (int64_t)a_at(Ap, KB, m, k) * w4_at(Bq, KB, n, k);
        acc[((size_t)m * G + g) * N + n] = (int32_t)s;
      }
}

/* fgm_gemm_q4g (amx_gemm.c:333-372) / fgm_gemm_q4g_vnni (vnni_gemm.c:291-322):
 * columns [n0*16, n1*16) of rows [0, M) of C, everything else untouched. */
void orc_gemm_q4g(int M, int N, int K, const int8_t *Ap, const float *a_scale,
                  const uint8_t *Bq, const uint16_t *b_scale, int group, float *C,
                  int ldc, int n0, int n1) {
  const int KB = K / 64, G = K / group;
  for (int m = 0; m < M; m++)
    for (int n = n0 * 16; n < n1 * 16; n++) {
      float c = 0.0f;
      for (int g = 0; g < G; g++) {
        int64_t s = 0;
        for (int k = g * group; k < (g + 1) * group; k++)
          s += (int64_t)a_at(Ap, KB, m, k) * w4_at(Bq, KB, n, k);
        c = fmaf((float)(int32_t)s, orc_f16_to_f32(b_scale[(size_t)g * N + n]), c);
      }
      C[(size_t)m * ldc + n] = c * a_scale[m];
    }
}

/* int32 accumulators of the int8 GEMM over the whole K: acc[m][n], [M][N]. */
void orc_gemm_q8c_acc(int M, int N, int K, const int8_t *Ap, const int8_t *B,
                      int32_t *acc, int n0, int n1) {
  const int KB = K / 64;
  for (int m = 0; m < M; m++)
    for (int n = n0 * 16; n < n1 * 16; n++) {
      int64_t s = 0;
      for (int k = 0; k < K; k++) s += (int64_t)a_at(Ap, KB, m, k) * w8_at(B, KB, n, k);
      acc[(size_t)m * N + n] = (int32_t)s;
    }
}

/* fgm_gemm_q8c (amx_gemm.c:444-475) / fgm_gemm_q8c_vnni (vnni_gemm.c:224-245). */
void orc_gemm_q8c(int M, int N, int K, const int8_t *Ap, const float *a_scale,
                  const int8_t *B, const float *b_scale, float *C, int ldc,
                  int n0, int n1) {
  const int KB = K / 64;
  (void)N;
  for (int m = 0; m < M; m++)
    for (int n = n0 * 16; n < n1 * 16; n++) {
      int64_t s = 0;
      for (int k = 0; k < K; k++) s += (int64_t)a_at(Ap, KB, m, k) * w8_at(B, KB, n, k);
      float bs = b_scale[n] * a_scale[m];
      C[(size_t)m * ldc + n] = (float)(int32_t)s * bs;
    }
}

/* Unpack an int4 tile blob to the int8 tile blob it encodes (inverse of
 * convert/quant.py:76-82 applied to the tile order of :96-107). */
void orc_unpack_q4_tiles(const uint8_t *Bq, size_t ntiles, int8_t *B8) {
  for (size_t t = 0; t < ntiles; t++)
    for (int r = 0; r < 16; r++)
      for (int i = 0; i < 64; i++) {
        int byte = Bq[t * Q4_TILE + (size_t)r * 32 + i % 32];
        B8[t * Q8_TILE + (size_t)r * 64 + i] =
            (int8_t)orc_nibble(i < 32 ? (byte & 0xF) : (byte >> 4));
      }
}

/* ------------------------------------------------- harness input generators
 * The reference's kernel harnesses draw their inputs from two small PRNGs.
 * Restating them lets the parity suite rebuild the exact inputs those
 * harnesses feed the reference kernels. */

/* bench/kernels/vnni_test.c:39-43: xorshift64, lo + state % (hi - lo + 1). */
void orc_fill_xorshift(uint64_t *state, int lo, int hi, size_t n, int32_t *out) {
  uint64_t rs = *state;
  for (size_t i = 0; i < n; i++) {
    rs ^= rs << 13; rs ^= rs >> 7; rs ^= rs << 17;
    out[i] = lo + (int)(rs % (uint64_t)(hi - lo + 1));
  }
  *state = rs;
}

/* bench/kernels/gemm_test.c:30-31: 32-bit LCG, lo + (state >> 16) % span. */
void orc_fill_lcg(uint32_t *state, int lo, int hi, size_t n, int32_t *out) {
  uint32_t rs = *state;
  for (size_t i = 0; i < n; i++) {
    rs = rs * 1103515245u + 12345u;
    out[i] = lo + (int)((rs >> 16) % (unsigned)(hi - lo + 1));
  }
  *state = rs;
}

/* Token choice after the LM head (fgm-serve/src/engine.rs:75-83,
 * fgm-bench/src/main.rs:201-209): scan ascending from (0, -inf), keep the
 * first strictly greater value. */
int orc_argmax(const float *v, int n) {
  int best = 0;
  float bv = -INFINITY;
  for (int i = 0; i < n; i++)
    if (v[i] > bv) {
      bv = v[i];
      best = i;
    }
  return best;
}

/* ====================================================================
 * Decode-chain glue (ops.c:55-147, :317-352) and the int8-KV attention
 * (ops.c:354-640, :641-665).  The reference runs these 16 floats at a time
 * (AVX-512) with a scalar libm tail; the restatement below reproduces the
 * vector arithmetic lane by lane, in the same order, so its outputs match
 * the compiled reference bit for bit wherever the reference does not call
 * libm (n a multiple of 16; rope always calls cosf/sinf).
 * ==================================================================== */

/* One lane of the reference's exp (ops.c:21-39): the Cephes range reduction
 * exp(x) = 2^n * exp(z), n = rint(x * log2 e), z = x - n*ln2 in two parts,
 * a degree-5 polynomial by fused multiply-adds, 2^n from the exponent bits.
 * Inputs are clamped to [-88, 88] first (max then min, so NaN -> -88). */
float orc_exp_lane(float x) {
  x = fmaxf(x, -88.0f);
  x = fminf(x, 88.0f);
  const float fx = rintf(x * 1.44269504088896341f);
  float z = fmaf(-fx, 0.693359375f, x);
  z = fmaf(-fx, -2.12194440e-4f, z);
  float y = 1.9875691500E-4f;
  y = fmaf(y, z, 1.3981999507E-3f);
  y = fmaf(y, z, 8.3334519073E-3f);
  y = fmaf(y, z, 4.1665795894E-2f);
  y = fmaf(y, z, 1.6666665459E-1f);
  y = fmaf(y, z, 5.0000001201E-1f);
  y = fmaf(y, z * z, z);
  y = y + 1.0f;
  const int32_t n = (int32_t)fx;
  const uint32_t bits = (uint32_t)(n + 127) << 23;
  float p2;
  memcpy(&p2, &bits, 4);
  return y * p2;
}

/* _mm512_reduce_add_ps as the reference's compiler lowers it: halves
 * (lanes i, i+8), then quarters (i, i+4), then pairs (i, i+2), then the
 * last two. */
float orc_reduce16(const float *a) {
  float t8[8], t4[4], t2[2];
  for (int i = 0; i < 8; i++) t8[i] = a[i] + a[i + 8];
  for (int i = 0; i < 4; i++) t4[i] = t8[i] + t8[i + 4];
  for (int i = 0; i < 2; i++) t2[i] = t4[i] + t4[i + 2];
  return t2[0] + t2[1];
}

/* ops.c:59-92: out = x * (mean(x^2) + eps)^-1/2 (* w when w != NULL). */
void orc_rmsnorm(float *out, const float *x, const float *w, int n, float eps) {
  float acc[16] = {0};
  int i = 0;
  for (; i + 16 <= n; i += 16)
    for (int j = 0; j < 16; j++) acc[j] = fmaf(x[i + j], x[i + j], acc[j]);
  float ss = orc_reduce16(acc);
  for (; i < n; i++) ss = fmaf(x[i], x[i], ss);
  const float inv = 1.0f / sqrtf(ss / (float)n + eps);
  for (i = 0; i < n; i++) out[i] = w ? (x[i] * inv) * w[i] : x[i] * inv;
}

/* ops.c:96-107: tanh-approximated GELU on one lane. */
static float gelu_lane(float x) {
  const float x3 = (x * x) * x;
  const float u = 0.7978845608028654f * fmaf(0.044715f, x3, x);
  const float e = orc_exp_lane(u + u);
  const float t = 1.0f - 2.0f / (e + 1.0f);
  return (0.5f * x) * (1.0f + t);
}

/* ops.c:119-131: out = gelu(gate) * up. */
void orc_gelu_mul(float *out, const float *gate, const float *up, int n) {
  int i = 0;
  for (; i + 16 <= n; i += 16)
    for (int j = 0; j < 16; j++) out[i + j] = gelu_lane(gate[i + j]) * up[i + j];
  for (; i < n; i++) {
    const float v = gate[i];
    out[i] = 0.5f * v * (1.0f + tanhf(0.7978845608028654f * (v + 0.044715f * v * v * v))) * up[i];
  }
}

/* ops.c:317-337 */
void orc_add(float *a, const float *b, int n) {
  for (int i = 0; i < n; i++) a[i] += b[i];
}
void orc_mul(float *a, const float *b, int n) {
  for (int i = 0; i < n; i++) a[i] *= b[i];
}
void orc_scale(float *a, float s, int n) {
  for (int i = 0; i < n; i++) a[i] *= s;
}

/* ops.c:340-352: x = cap * tanh(x / cap), tanh from the exp lane. */
void orc_softcap(float *x, int n, float cap) {
  const float ci = 1.0f / cap;
  int i = 0;
  for (; i + 16 <= n; i += 16)
    for (int j = 0; j < 16; j++) {
      const float u = x[i + j] * ci;
      const float e = orc_exp_lane(u + u);
      x[i + j] = cap * (1.0f - 2.0f / (e + 1.0f));
    }
  for (; i < n; i++) x[i] = cap * tanhf(x[i] / cap);
}

/* ops.c:135-147: half-split rotary embedding of n_heads heads in place.
 * fused: the two products-and-sum as fused multiply-adds (a build that
 * contracts the reference's scalar expressions) or as separate roundings. */
void orc_rope(float *x, int n_heads, int head_dim, const float *inv_freq, int pos, int fused) {
  const int h = head_dim / 2;
  for (int j = 0; j < h; j++) {
    const float a = (float)pos * inv_freq[j];
    const float c = cosf(a), s = sinf(a);
    for (int hh = 0; hh < n_heads; hh++) {
      float *p = x + (size_t)hh * head_dim;
      const float lo = p[j], hi = p[j + h];
      if (fused) {
        p[j] = fmaf(lo, c, -(hi * s));
        p[j + h] = fmaf(hi, c, lo * s);
      } else {
        p[j] = lo * c - hi * s;
        p[j + h] = hi * c + lo * s;
      }
    }
  }
}

/* ops.c:653-660: one int8 V row into the slot-interleaved cache. */
void orc_store_v_t(int8_t *vt, const int8_t *src, int n, int slot) {
  int8_t *dst = vt + (size_t)(slot >> 2) * n * 4 + (slot & 3);
  for (int j = 0; j < n; j++) dst[(size_t)j * 4] = src[j];
}

/* ops.c:378-640 (fgm_attend_q8_heads), heads [h0, h1) of one query row
 * against positions [start, end) of an int8 KV cache: K [slot][kv_heads *
 * head_dim] with per-slot scales ks, V slot-interleaved (orc_store_v_t) with
 * scales vs; ring = 0 for a linear cache, else slots are positions mod ring.
 *  - Q per head: s = max|q| / 127, q8 = clamp(rint(q * 127/max), -127, 127);
 *  - score_t = (float)(q8 . k_t) * s * ks_t  (the reference's biased VNNI
 *    dot minus its correction is exactly q8 . k_t);
 *  - softmax over 16-position chunks with the exp lane, sums per lane then
 *    reduced, the tail with libm expf; inv = 1 / sum;
 *  - weight w_t = score_t * inv * vs_t, quantised to 16 bits of wmax:
 *    iw = (int)(w_t * 65535/wmax + 0.5), split into hi / lo bytes;
 *  - out = (float)(256 * sum hi_t v_t + sum lo_t v_t) * (wmax / 65535).
 * scratch holds (end - start) floats. */
void orc_attend_q8_heads(float *out, const float *q, const int8_t *kc, const float *ks,
                         const int8_t *vc, const float *vs, int n_heads, int kv_heads,
                         int head_dim, int start, int end, float *scratch, int h0, int h1,
                         int ring) {
  const int kvd = kv_heads * head_dim, grp = n_heads / kv_heads;
  for (int h = h0; h < h1; h++) {
    const float *qh = q + (size_t)h * head_dim;
    const int kvh = h / grp;
    float *sc = scratch;
    int8_t qq[512];
    float qamax = 0.0f;
    for (int i = 0; i < head_dim; i++) {
      const float a = fabsf(qh[i]);
      if (a > qamax) qamax = a;
    }
    const float qscale = qamax / 127.0f;
    const float qinv = qamax > 0.0f ? 127.0f / qamax : 0.0f;
    for (int i = 0; i < head_dim; i++) {
      int v = (int)lrintf(qh[i] * qinv);
      v = v > 127 ? 127 : (v < -127 ? -127 : v);
      qq[i] = (int8_t)v;
    }
    float mx = -INFINITY;
    for (int t = start; t < end; t++) {
      const int sl = ring ? t % ring : t;
      const int8_t *kp = kc + (size_t)sl * kvd + (size_t)kvh * head_dim;
      int32_t dot = 0;
      for (int i = 0; i < head_dim; i++) dot += (int32_t)kp[i] * (int32_t)qq[i];
      const float s = (float)dot * qscale * ks[sl];
      sc[t - start] = s;
      if (s > mx) mx = s;
    }
    const int n = end - start;
    float lanes[16] = {0};
    int u = 0;
    for (; u + 16 <= n; u += 16)
      for (int j = 0; j < 16; j++) {
        const float e = orc_exp_lane(sc[u + j] - mx);
        sc[u + j] = e;
        lanes[j] = lanes[j] + e;
      }
    float sum = orc_reduce16(lanes);
    for (; u < n; u++) {
      sc[u] = expf(sc[u] - mx);
      sum += sc[u];
    }
    const float inv = 1.0f / sum;
    float wmax = 0.0f;
    for (int t = start; t < end; t++) {
      const float w = sc[t - start] * inv * vs[ring ? t % ring : t];
      if (w > wmax) wmax = w;
    }
    float *oh = out + (size_t)h * head_dim;
    if (!(wmax > 0.0f)) {
      for (int i = 0; i < head_dim; i++) oh[i] = 0.0f;
      continue;
    }
    const float wq_scale = wmax / 65535.0f, wq_inv = 65535.0f / wmax;
    int32_t acc_hi[512], acc_lo[512];
    for (int i = 0; i < head_dim; i++) acc_hi[i] = acc_lo[i] = 0;
    for (int t = start; t < end; t++) {
      const int sl = ring ? t % ring : t;
      int iw = (int)(sc[t - start] * inv * vs[sl] * wq_inv + 0.5f);
      if (iw > 65535) iw = 65535;
      if (iw < 0) iw = 0;
      const int hi = iw >> 8, lo = iw & 255;
      const int8_t *vrow = vc + ((size_t)(sl >> 2) * kvd + (size_t)kvh * head_dim) * 4 + (sl & 3);
      for (int i = 0; i < head_dim; i++) {
        acc_hi[i] += hi * (int32_t)vrow[(size_t)i * 4];
        acc_lo[i] += lo * (int32_t)vrow[(size_t)i * 4];
      }
    }
    for (int i = 0; i < head_dim; i++)
      oh[i] = (float)(int32_t)(((uint32_t)acc_hi[i] << 8) + (uint32_t)acc_lo[i]) * wq_scale;
  }
}
