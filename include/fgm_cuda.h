/*
 * fgm_cuda.h -- C ABI of the B200 (sm_100a) backend for fastgemma's quantised
 * GEMM hot path.  Implemented by libfgm_cuda.so (fastgemma_b200/csrc).
 *
 * The reference binds its CPU kernels through the `extern "C"` block of
 * crates/fgm-kernels/src/lib.rs:13-80 and dispatches on `Backend`
 * (lib.rs:86-138).  This header is what a third backend, `Backend::Cuda`,
 * binds.  Reference paths are relative to the fastgemma project root.
 *
 * Conventions shared by every entry point:
 *  - Return 0 on success, a negative FGM_CUDA_E* code on failure.  Nothing
 *    aborts the process; fgm_cuda_last_error() describes the last failure on
 *    the calling thread.  (The reference returns void and leaves misuse
 *    undefined; lib.rs:177-178 / :203-204 only debug-assert the shapes.)
 *  - Shape contract, checked on every call (EINVAL otherwise): K > 0,
 *    K % 64 == 0, K <= 65536; N > 0, N % 16 == 0; M >= 0;
 *    0 <= n0 <= n1 <= N/16 and (n1 - n0) % 4 == 0 (n-blocks of 16 columns,
 *    stepped in fours as pool.rs:121-124 splits them); ldc >= N;
 *    for int4: group > 0, group % 64 == 0, K % group == 0.
 *  - A is tile-packed activations [ceil(M/16)][K/64][16][64] int8 with zero
 *    padding rows (ops.c:279-290); a_scale is f32 [M].
 *  - int4 weights: the .fgm q4g blob, N*K/2 bytes, tiles [N/16][K/64] of
 *    512 bytes, nibble-packed (convert/quant.py:76-107); scales f16
 *    [K/group][N] passed as raw uint16 (model.rs:182).
 *  - int8 weights: the .fgm q8c blob, N*K bytes, tiles [N/16][K/64] of 1024
 *    bytes [k/4][n][k%4]; scales f32 [N] (convert/quant.py:110-117).
 *  - C is f32 row-major with leading dimension ldc; only rows [0, M) and
 *    columns [n0*16, n1*16) are written (amx_gemm.c:333-372 contract).
 *  - Arithmetic is bit-exact with the reference kernels: int32 accumulators
 *    per scale group, then for int4 C = a_scale[m] * fold_g fma(acc_g, s_g, .)
 *    in ascending group order, for int8 C = acc * (b_scale[n] * a_scale[m]).
 */
#ifndef FGM_CUDA_H
#define FGM_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  FGM_CUDA_OK = 0,
  FGM_CUDA_EINVAL = -1,   /* argument outside the shape contract */
  FGM_CUDA_ENODEV = -2,   /* no sm_100 device, or the device is unusable */
  FGM_CUDA_ERUNTIME = -3, /* a CUDA runtime call or kernel launch failed */
  FGM_CUDA_ENOMEM = -4,   /* device or pinned-host allocation failed */
  FGM_CUDA_ETIMEOUT = -5  /* a bounded device-side wait gave up */
};

/* ------------------------------------------------------------ probe / setup */

/* 1 if a compute-capability 10.x device is visible, else 0.  The CUDA analogue
 * of fgm_cpu_has_amx / fgm_cpu_has_avx512_vnni (vnni_gemm.c:61-80), which
 * backend() consults before choosing (lib.rs:112-138). */
int fgm_cuda_available(void);

/* Bind the library to `device` (-1: FGM_CUDA_DEVICE or the current device).
 * Optional: every entry point initialises lazily.  No reference counterpart
 * beyond fgm_amx_init (amx_gemm.c:40), the per-thread capability grant. */
int fgm_cuda_init(int device);

/* Text of the last failure on the calling thread ("" if none). */
const char *fgm_cuda_last_error(void);

/* Number of kernels this library has launched since load (instrumentation). */
uint64_t fgm_cuda_launch_count(void);

/* Wait for the current device, then report whether any kernel of this library
 * gave up on a bounded wait since the last call (FGM_CUDA_ETIMEOUT, flag
 * cleared) -- every device-side wait has a time limit instead of spinning
 * forever.  No reference counterpart (the CPU kernels never wait). */
int fgm_cuda_device_status(void);

/* ---------------------------------------------- drop-ins, host pointers
 * Same argument lists as the reference symbols, plus a status return.  All
 * pointers are HOST pointers; the call is synchronous like the reference's.
 * Weights (Bq/B and their scales) registered with fgm_cuda_register() are
 * used from their resident device copy -- the intended mode, matching the
 * reference's immutable mmap'd blobs (model.rs:98-103).  Unregistered weights
 * are still correct: they are uploaded for that call alone, never cached, so
 * a host buffer reused for other data can not be served stale.  Activations
 * and C cross the bus on every call.  Serialised internally: concurrent
 * callers are safe but do not overlap. */

/* replaces fgm_gemm_q4g (amx_gemm.c:333) and fgm_gemm_q4g_vnni
 * (vnni_gemm.c:291); Rust binding lib.rs:21-25 */
int fgm_gemm_q4g_cuda(int M, int N, int K, const int8_t *A, const float *a_scale,
                      const uint8_t *Bq, const uint16_t *b_scale, int group,
                      float *C, int ldc, int n0, int n1);

/* replaces fgm_gemm_q8c (amx_gemm.c:444) and fgm_gemm_q8c_vnni
 * (vnni_gemm.c:224); Rust binding lib.rs:26-30 */
int fgm_gemm_q8c_cuda(int M, int N, int K, const int8_t *A, const float *a_scale,
                      const int8_t *B, const float *b_scale, float *C, int ldc,
                      int n0, int n1);

/* Gemm::run (crates/fgm-core/src/forward.rs:128-158) on this backend: the
 * pair Pool::prep + Pool::gemm (pool.rs:285-311) that every linear layer
 * issues, as one call.  src [M, lda] f32 host rows are rotated (hsz), quantised
 * and packed on the device, multiplied over all N columns, and C [M, ldc]
 * comes back to the host.  N % 64 == 0. */
int fgm_linear_q4g_cuda(const float *src, int lda, int hsz, int M, int N, int K,
                        const uint8_t *Bq, const uint16_t *b_scale, int group,
                        float *C, int ldc);
int fgm_linear_q8c_cuda(const float *src, int lda, int hsz, int M, int N, int K,
                        const int8_t *B, const float *b_scale, float *C, int ldc);

/* replaces fgm_prep_rows (ops.c:293-314); Rust binding lib.rs:17-20.
 * src [m, lda] f32 rows -> rot [m, k] f32 (rotated copy), qa [m, k] int8,
 * qs [m] f32 scales, pa tile-packed.  Rows [r0, r1), r0 % 16 == 0,
 * k % 64 == 0, hsz 0 or a power of two dividing k.  rot and qa may be NULL. */
int fgm_prep_rows_cuda(const float *src, int lda, float *rot, int8_t *qa,
                       float *qs, int8_t *pa, int m, int k, int hsz, int r0,
                       int r1);

/* replaces fgm_quant_act (ops.c:181-204); Rust binding lib.rs:54 */
int fgm_quant_act_cuda(const float *x, int rows, int k, int8_t *q, float *scale);

/* replaces fgm_fwht (ops.c:153-175); Rust binding lib.rs:53.  n % hsz == 0. */
int fgm_fwht_cuda(float *x, int n, int hsz);

/* replaces fgm_pack_a (ops.c:279-290); Rust binding lib.rs:16 */
int fgm_pack_a_cuda(int M, int K, const int8_t *A, int8_t *Ap);

/* ---------------------------------------------------------- weight registry
 * Device-resident copies of immutable host weight blobs, keyed by host
 * address.  The reference needs none: its kernels read the mmap directly
 * (model.rs:120-128). */

/* Upload `bytes` at `host` once (no-op if already registered with the same
 * size; EINVAL if registered with another size).  The blob must not change
 * while registered: the host-pointer entry points serve the device copy. */
int fgm_cuda_register(const void *host, size_t bytes);
/* Drop the device copy (and any derived operand copy) of `host`. */
int fgm_cuda_unregister(const void *host);
/* Device address of a registered blob, or NULL. */
const void *fgm_cuda_lookup(const void *host);
/* Total device bytes held by the registry. */
size_t fgm_cuda_registry_bytes(void);

/* ------------------------------------- device pointers, asynchronous
 * Same contracts with every buffer in device memory; work is enqueued on
 * `stream` (a cudaStream_t; NULL = the legacy default stream) and the call
 * returns without waiting.  These are the entry points a GPU-resident forward
 * pass uses. */

int fgm_cuda_gemm_q4g(int M, int N, int K, const int8_t *A, const float *a_scale,
                      const uint8_t *Bq, const uint16_t *b_scale, int group,
                      float *C, int ldc, int n0, int n1, void *stream);

int fgm_cuda_gemm_q8c(int M, int N, int K, const int8_t *A, const float *a_scale,
                      const int8_t *B, const float *b_scale, float *C, int ldc,
                      int n0, int n1, void *stream);

/* fgm_cuda_gemm_q4g / fgm_cuda_gemm_q8c that also warm L2 for the launch
 * that follows: once this GEMM's own weight stream is queued, its CTAs
 * prefetch [next_w, next_w + next_w_bytes) and [next_s, next_s +
 * next_s_bytes) (16-byte aligned; a null pointer or 0 bytes = none) into L2,
 * so HBM keeps streaming across the kernel boundary and the next decode GEMM
 * finds its weights on chip.  The prefetch has no completion and changes no
 * result.  A decode forward knows its layer order, so it passes the next
 * projection's tile blob and scales.  No reference counterpart: the
 * reference's CPU GEMMs (amx_gemm.c:333-475) stream from DRAM per call. */
int fgm_cuda_gemm_q4g_warm(int M, int N, int K, const int8_t *A, const float *a_scale,
                           const uint8_t *Bq, const uint16_t *b_scale, int group, float *C,
                           int ldc, int n0, int n1, const void *next_w, size_t next_w_bytes,
                           const void *next_s, size_t next_s_bytes, void *stream);

int fgm_cuda_gemm_q8c_warm(int M, int N, int K, const int8_t *A, const float *a_scale,
                           const int8_t *B, const float *b_scale, float *C, int ldc, int n0,
                           int n1, const void *next_w, size_t next_w_bytes, const void *next_s,
                           size_t next_s_bytes, void *stream);

/* One projection of fgm-core's Gemm::run (forward.rs:128-158) on device
 * buffers: f32 rows src [M][lda] are rotated (hsz), quantised per row and
 * multiplied into C [M][ldc], columns [n0*16, n1*16), on `stream`.  The
 * device form of fgm_linear_q4g_cuda / fgm_linear_q8c_cuda: the prep kernel
 * writes the int8 rows to stream-ordered temporary memory, then the GEMM
 * (tcgen05 for prepared int8 weights and M >= 64).  Same contracts as
 * fgm_cuda_gemm_* and fgm_cuda_prep_rows. */
int fgm_cuda_linear_q4g(const float *src, int lda, int hsz, int M, int N, int K,
                        const uint8_t *Bq, const uint16_t *b_scale, int group,
                        float *C, int ldc, int n0, int n1, void *stream);
int fgm_cuda_linear_q8c(const float *src, int lda, int hsz, int M, int N, int K,
                        const int8_t *B, const float *b_scale, float *C, int ldc,
                        int n0, int n1, void *stream);

/* Tensor-core operand copy of a device-resident int8 weight (the .fgm tiles
 * at B, N x K) as a row-major [N][K] matrix, plus its TMA descriptor, kept
 * until fgm_cuda_q8c_release(B).  Once a weight is prepared,
 * fgm_cuda_gemm_q8c / _acc with M >= 64 (FGM_CUDA_TC_MIN_M) run on the
 * tcgen05 kernel (tile-packed A is first copied to row-major form in
 * stream-ordered temporary memory); unprepared weights and small M use the
 * streaming kernel.  Host-pointer entry points prepare registered weights on
 * first large-M use.  The copy costs N*K device bytes.  No reference
 * counterpart: the AMX kernel consumes the tiles as they are
 * (amx_gemm.c:375-410). */
int fgm_cuda_q8c_prepare(const int8_t *B, int N, int K, void *stream);

/* Prefill form of fgm_cuda_gemm_q8c: activations as the quantiser's row-major
 * int8 matrix A [M][lda] (fgm_quant_act's q, ops.c:181-204; lda >= K,
 * lda % 16 == 0) instead of the tile-packed copy, weight prepared with
 * fgm_cuda_q8c_prepare (EINVAL otherwise).  Always the tcgen05 kernel. */
int fgm_cuda_gemm_q8c_rows(int M, int N, int K, const int8_t *A, int lda,
                           const float *a_scale, const int8_t *B,
                           const float *b_scale, float *C, int ldc, int n0, int n1,
                           void *stream);
int fgm_cuda_q8c_release(const int8_t *B);

/* fgm_cuda_gemm_q8c on the tcgen05 kernel without any device allocation, for
 * callers that may not allocate once serving (a fully reserved HBM budget, or
 * a host language with no say over the CUDA memory pools).  No reference
 * counterpart: the reference CPU kernels read the tile-packed A in place.
 * The tile-packed A is copied to row-major form in a fixed 4 MiB device
 * buffer owned by the library instead of stream-ordered temporary memory:
 * M*K > 4194304 is rejected with EINVAL.  The weight must be prepared with
 * fgm_cuda_q8c_prepare (EINVAL otherwise); any M >= 1 runs the tensor-core
 * kernel.  The first call on each device is set-up (it resolves the buffer's
 * address and the device's status word): make it before any stream capture.
 * One buffer per device: calls that overlap in time (different streams or
 * host threads) race on it; calls on one stream are ordered.  The buffer is
 * a file-scope device array, so every device on which this library's kernels
 * load holds its 4 MiB until the process exits. */
int fgm_cuda_gemm_q8c_noalloc(int M, int N, int K, const int8_t *A, const float *a_scale,
                              const int8_t *B, const float *b_scale, float *C, int ldc,
                              int n0, int n1, void *stream);

/* rot and qa may be NULL (not written). */
int fgm_cuda_prep_rows(const float *src, int lda, float *rot, int8_t *qa,
                       float *qs, int8_t *pa, int m, int k, int hsz, int r0,
                       int r1, void *stream);

/* int32 accumulators of the int4 product, acc [M][K/group][N]:
 * acc[m][g][n] = sum over group g of A[m][k] * W[n][k], columns
 * [n0*16, n1*16).  Same kernel as fgm_cuda_gemm_q4g with the f32 epilogue
 * replaced by a raw store, for bit-exact accumulator checks.  No reference
 * counterpart: the reference never exposes its int32 lanes. */
int fgm_cuda_gemm_q4g_acc(int M, int N, int K, const int8_t *A, const uint8_t *Bq,
                          int group, int32_t *acc, int n0, int n1, void *stream);

/* int32 accumulators of the int8 product over all K, acc [M][N]. */
int fgm_cuda_gemm_q8c_acc(int M, int N, int K, const int8_t *A, const int8_t *B,
                          int32_t *acc, int n0, int n1, void *stream);

/* ------------------------------------------------------ decode work list
 * A decode step's sequence of Gemm::run calls (fgm-core/src/forward.rs:128-158
 * per projection, each a prep of its f32 input and an int4 or int8 GEMM) as
 * ONE persistent kernel launch per run: every SM streams the weights of its
 * share of every item through shared memory without stopping at item
 * boundaries, and an item that reads another item's output waits on that
 * item's completion counter (device-side, bounded) instead of a kernel
 * boundary.  Each GEMM item computes exactly fgm_cuda_gemm_q4g /
 * fgm_cuda_gemm_q8c over its column range, each prep item exactly
 * fgm_cuda_prep_rows over rows [0, M) -- bit-identical outputs.  (A prep
 * that depends on no other entry leaves the padding rows of its 16-row
 * block as they are; in the list's GEMMs padding rows reach only outputs
 * that are not stored.)  The preps that depend on no entry are prepared at
 * the start of the run by all SMs together, after each SM has started its
 * weight stream.  No reference counterpart: the reference
 * runs its projections one call at a time (pool.rs:126-145).
 *
 * A list is created once (validation, schedule, activation TMA descriptors,
 * its device-side descriptors and counters: the only allocations) and run any
 * number of times; every pointer in it stays fixed for the list's lifetime.
 * Contract per entry (EINVAL otherwise), with 1 <= M <= 16 for the whole list:
 *  - FGM_CUDA_WORK_Q4G / _Q8C: weight [N, K] in the .fgm layout, N % 16 == 0,
 *    K % 512 == 0 (int4) or K % 256 == 0 (int8), K <= 16384; output columns
 *    [n0*16, n1*16), 0 <= n0 < n1 <= N/16, C[m*ldc + n] with ldc >= n1*16;
 *    int4 group in {64, 128, 256, 512} dividing K; A (tile-packed, one 16-row
 *    block; rows past M reach no stored output), B and int4 scales 16-byte aligned, int8
 *    scales 4-byte aligned.
 *  - FGM_CUDA_WORK_PREP: f32 rows src[m*lda + k], K % 128 == 0, lda >= K,
 *    lda % 4 == 0, src 16-byte aligned; hsz 0 or a power of two <= 128
 *    dividing K (the FWHT block, ops.c:153-175); outputs pa (the packed 16-row
 *    block, packed_a_len(M, K) bytes, 4-byte aligned) and qs [M].
 *  - Prep sources and GEMM outputs may be page-locked host memory (read and
 *    written by the kernel through their device mapping, so one run moves a
 *    step's inputs and results across the host link itself); every other
 *    buffer must be device memory.  Pageable host memory is rejected.
 *  - deps: up to two indices of EARLIER entries whose outputs this entry
 *    reads (-1: none).  Inputs written before the run (earlier kernels on the
 *    stream) need no entry.  Entries that write memory another entry reads or
 *    writes must be ordered by deps; the kernel does not check it.
 * Runs of one list must not overlap in time (they share its counters). */
enum { FGM_CUDA_WORK_Q4G = 0, FGM_CUDA_WORK_Q8C = 1, FGM_CUDA_WORK_PREP = 2 };

typedef struct fgm_cuda_work {
  int kind;               /* FGM_CUDA_WORK_* */
  int N, K, group;        /* GEMM: weight shape, int4 scale group; PREP: K = row length */
  int n0, n1, ldc;        /* GEMM: output n-blocks [n0, n1), C row pitch */
  int lda, hsz;           /* PREP: source row pitch (floats), FWHT block (0: none) */
  int deps[2];            /* earlier entries this one waits for (-1: none) */
  const int8_t *A;        /* GEMM: tile-packed activations */
  const float *a_scale;   /* GEMM: [M] */
  const void *B;          /* GEMM: weight blob (int4 q4g or int8 q8c) */
  const void *b_scale;    /* GEMM: f16 [K/group][N] (int4) or f32 [N] (int8) */
  float *C;               /* GEMM output */
  const float *src;       /* PREP input rows */
  int8_t *pa;             /* PREP: packed rows out */
  float *qs;              /* PREP: row scales out */
} fgm_cuda_work;

/* Validate and schedule `n` entries for batch size M on the current device;
 * *list receives the handle. */
int fgm_cuda_worklist_create(int M, const fgm_cuda_work *items, int n, void **list);
/* One launch of the whole list on `stream` (NULL: the default stream). */
int fgm_cuda_worklist_run(void *list, void *stream);
/* Free a list (waits for the device first). */
int fgm_cuda_worklist_destroy(void *list);

/* ------------------------------------------- decode-chain glue, attention
 * The operations between the GEMMs of the reference's decode forward pass
 * (fgm-core/src/forward.rs:469-654), on device buffers and a stream, as
 * fgm-kernels computes them (crates/fgm-kernels/csrc/ops.c).  Bit-identical
 * to the reference for row lengths that are multiples of 16; the reference's
 * libm pieces (scalar tails, rope's cos / sin, the softmax tail's exp) are
 * evaluated in double precision and rounded once. */

/* ops.c:59-92 (fgm_rmsnorm; fgm_rmsnorm_noscale when w is NULL): each of
 * `rows` rows of n: out = x * (mean(x^2) + eps)^-1/2 (* w). n <= 49152. */
int fgm_cuda_rmsnorm(float *out, const float *x, const float *w, int rows, int n, float eps,
                     void *stream);

/* ops.c:119-131 (fgm_gelu_mul): out = gelu_tanh(gate) * up over rows of n. */
int fgm_cuda_gelu_mul(float *out, const float *gate, const float *up, int rows, int n,
                      void *stream);

/* ops.c:317-337 (fgm_add, fgm_mul, fgm_scale) over n floats, in place. */
int fgm_cuda_add(float *a, const float *b, size_t n, void *stream);
int fgm_cuda_mul(float *a, const float *b, size_t n, void *stream);
int fgm_cuda_scale(float *a, float s, size_t n, void *stream);

/* ops.c:340-352 (fgm_softcap): x = cap * tanh(x / cap) over rows of n. */
int fgm_cuda_softcap(float *x, int rows, int n, float cap, void *stream);

/* ops.c:135-147 (fgm_rope): half-split rotary embedding of n_heads heads,
 * in place, for `rows` rows (row r at x + r*x_ld) at positions pos[r] (a
 * device array). */
int fgm_cuda_rope(float *x, int x_ld, int rows, int n_heads, int head_dim, const float *inv_freq,
                  const int *pos, void *stream);

/* Rope bit-identical to the reference: its cos / sin are this host's libm
 * cosf / sinf of (float)pos * inv_freq[j] (ops.c:137-139), which the device
 * cannot reproduce call for call.  fgm_cuda_rope_table fills, on the host
 * (no device work), cs[p * head_dim + j] = cosf and cs[p * head_dim +
 * head_dim/2 + j] = sinf for positions p in [0, positions) and j <
 * head_dim/2.  Copied to the device, the table feeds fgm_cuda_rope_cs and
 * fgm_cuda_qkv_post_cs; a row whose position lies outside [0, positions)
 * falls back to the device evaluation of fgm_cuda_rope. */
int fgm_cuda_rope_table(float *cs, int positions, int head_dim, const float *inv_freq);
int fgm_cuda_rope_cs(float *x, int x_ld, int rows, int n_heads, int head_dim,
                     const float *inv_freq, const float *cs, int positions, const int *pos,
                     void *stream);

/* ops.c:181-204, :641-644 (fgm_quant_act, fgm_quant_kv): rows of k f32 to
 * int8 with one scale per row (k % 64 == 0). */
int fgm_cuda_quant_act(const float *x, int rows, int k, int8_t *q, float *scale, void *stream);

/* ops.c:653-660 (fgm_store_v_t): for each of `rows` caches (vt +
 * r*vt_stride bytes), store the int8 V row src + r*src_ld (n bytes) at
 * `slot` of the slot-interleaved layout vt[((slot/4)*n + j)*4 + slot%4]. */
int fgm_cuda_store_v_t(int8_t *vt, size_t vt_stride, const int8_t *src, int src_ld, int rows,
                       int n, int slot, void *stream);

/* ops.c:378-640 (fgm_attend_q8 / fgm_attend_q8_heads): for each of `rows`
 * query rows (its own KV cache at the given per-row strides, in elements),
 * all n_heads heads of q + r*q_ld attend to positions [start, end) of an
 * int8 cache: K [slot][kv_heads*head_dim] with scales ks [slot], V in the
 * store_v_t layout (holding whole groups of four slots) with scales vs.
 * ring = 0: slot = position; ring > 0: slot = position % ring and the
 * window must not be longer than the ring.  head_dim % 64 == 0, <= 512; at
 * most 16 query heads per KV head; the caches and their row strides 4-byte
 * aligned (16-byte aligned ones copy faster). */
int fgm_cuda_attend_q8(float *out, int out_ld, const float *q, int q_ld, const int8_t *kc,
                       size_t kc_stride, const float *ks, size_t ks_stride, const int8_t *vt,
                       size_t vt_stride, const float *vs, size_t vs_stride, int rows, int n_heads,
                       int kv_heads, int head_dim, int start, int end, int ring, void *stream);

/* ------------------------------------------- fused glue of a decode step
 * Each entry is one launch for a run of reference operations between two
 * GEMMs, bit-identical to calling the entries above one after the other.
 *
 * fgm_cuda_norm_prep (forward.rs:476-480, :625-654): when proj is not null,
 * h += rmsnorm(proj, w_post) for each row (ops.c:59-92 then :317-321; h
 * updated in place); then the packed int8 rows (and scales) of
 * rmsnorm(h, w_pre) for the next GEMM, as fgm_cuda_prep_rows with hsz 0.
 * Rows of n floats (n % 64 == 0, n <= 12288; h, proj and the norm weights
 * 16-byte aligned);
 * pa holds (rows rounded up to 16) x n bytes, the padding rows are
 * zero-filled. */
int fgm_cuda_norm_prep(float *h, const float *proj, const float *w_post, const float *w_pre,
                       int rows, int n, float eps, float *qs, int8_t *pa, void *stream);

/* fgm_cuda_gelu_mul_prep (forward.rs:641-643): the down projection's packed
 * rows of gelu(gate) * up (ops.c:119-131 per row of n, n % 64 == 0; gate
 * and up rows ld floats apart, so one fused [gate | up] GEMM output serves
 * as both), and the f32 product in act [rows][n] when act is not null (all
 * 16-byte aligned, ld % 4 == 0). */
int fgm_cuda_gelu_mul_prep(const float *gate, const float *up, int ld, int rows, int n,
                           float *act, float *qs, int8_t *pa, void *stream);

/* fgm_cuda_qkv_post (forward.rs:482-545): for each row r, rmsnorm of every
 * query head (q_norm) and key head (k_norm) followed by rope at pos[r]
 * (ops.c:135-147), rmsnorm without scale of every value head, all in place
 * in q (rows q_ld floats apart), k and v (rows kv_ld apart); then
 * the key and value rows quantised to int8 with one scale each (ops.c:
 * 181-204) into row r's caches at slot pos[r] (pos[r] % ring when ring >
 * 0): kc + r*kc_stride [slot][kv_heads*head_dim], ks + r*ks_stride [slot],
 * V into vt + r*vt_stride in the store_v_t layout, vs + r*vs_stride [slot].
 * Each cache holds cap slots (0 < ring <= cap); a row whose slot falls
 * outside [0, cap) writes no cache entry.
 * head_dim % 4 == 0, at most 48 heads in all, q, k and v 16-byte aligned,
 * q_ld and kv_ld multiples of 4. */
int fgm_cuda_qkv_post(float *q, int q_ld, float *k, float *v, int kv_ld, int rows, int n_heads,
                      int kv_heads, int head_dim, const float *q_norm, const float *k_norm, float eps,
                      const float *inv_freq, const int *pos, int ring, int cap, int8_t *kc,
                      size_t kc_stride, float *ks, size_t ks_stride, int8_t *vt, size_t vt_stride,
                      float *vs, size_t vs_stride, void *stream);
/* fgm_cuda_qkv_post with rope's cos / sin from a device copy of
 * fgm_cuda_rope_table (positions entries; see fgm_cuda_rope_cs). */
int fgm_cuda_qkv_post_cs(float *q, int q_ld, float *k, float *v, int kv_ld, int rows,
                         int n_heads, int kv_heads, int head_dim, const float *q_norm,
                         const float *k_norm, float eps, const float *inv_freq, const float *cs,
                         int positions, const int *pos, int ring, int cap, int8_t *kc,
                         size_t kc_stride, float *ks, size_t ks_stride, int8_t *vt,
                         size_t vt_stride, float *vs, size_t vs_stride, void *stream);

/* ------------------------------------------------------------ row argmax
 * The token choice that follows the LM head (fgm-serve/src/engine.rs:75-83,
 * :297-302): per row the first index of the largest value, NaN never
 * chosen, 0 when nothing exceeds -inf.  Split so a column-sharded LM head
 * exchanges a few pairs instead of the logits:
 * fgm_cuda_argmax_partials writes, for each row m of C [M][ldc] (columns
 * [0, N), reported as col0 + column), fgm_cuda_argmax_parts(N) partial
 * (value, index) pairs at vals/idx[m * parts + p] (index -1: nothing above
 * -inf); fgm_cuda_argmax_merge folds P pairs per row (row m's at m * P ...)
 * into out[m].  Partials from several ranks concatenated per row merge the
 * same way. */
int fgm_cuda_argmax_parts(int N);
int fgm_cuda_argmax_partials(const float *C, int M, int N, int ldc, int col0, float *vals,
                             int32_t *idx, void *stream);
int fgm_cuda_argmax_merge(const float *vals, const int32_t *idx, int M, int P, int32_t *out,
                          void *stream);

/* ----------------------------------- column-sharded GEMM, fused gather
 * The large-N products (the LM head, forward.rs:301, :687) split by output
 * columns over the GPUs of one node.  No reference counterpart: the
 * reference splits the same column ranges over CPU threads (pool.rs:110-124)
 * and needs no exchange.
 *
 * Peer memory: each rank allocates its buffers with fgm_cuda_ipc_alloc
 * (zeroed), exports FGM_CUDA_IPC_HANDLE_BYTES-byte handles, and opens the
 * other ranks' handles (same node). */
#define FGM_CUDA_IPC_HANDLE_BYTES 64
int fgm_cuda_ipc_alloc(size_t bytes, void **dev_ptr);
int fgm_cuda_ipc_free(void *dev_ptr);
int fgm_cuda_ipc_handle(const void *dev_ptr, void *handle);
int fgm_cuda_ipc_open(const void *handle, void **dev_ptr);
int fgm_cuda_ipc_close(void *dev_ptr);

/* This rank's share of a column-sharded int4 decode GEMM with the all-gather
 * fused into it: Bq/b_scale hold this rank's N columns (a shard of the .fgm
 * blob), which land at columns [col0, col0 + N) of every rank's output
 * out[q] -- two buffers per rank, slot s at out[q] + s*slot_floats, each
 * [M][ldc] f32 (M <= 16) -- locally and over NVLink into each peer.  sig[q]
 * are the ranks' signal words (FGM_CUDA_GATHER_SIG_BYTES, zeroed, from
 * fgm_cuda_ipc_alloc).  Collective: every rank makes the same sequence of
 * calls; call c uses slot c % 2, counted on the device (a rank's own signal
 * words hold its completed calls), so the arguments never change between
 * calls and a sequence of calls can be replayed from a CUDA graph.  When the
 * kernel completes on `stream`, slot c % 2 of out[rank] holds all ranks'
 * columns; it stays valid until the call after next.  Words 8..10 of a rank's
 * signal block hold %globaltimer stamps of its last call (start, own columns
 * pushed, every rank's columns arrived).  Every cross-GPU wait is bounded
 * (2 s, then fgm_cuda_device_status reports FGM_CUDA_ETIMEOUT; the ranks'
 * counters may then disagree: make new buffers). */
#define FGM_CUDA_GATHER_SIG_BYTES 128
int fgm_cuda_gemm_q4g_gather(int M, int N, int K, const int8_t *A, const float *a_scale,
                             const uint8_t *Bq, const uint16_t *b_scale, int group,
                             int col0, int ldc, void *const *out,
                             unsigned long long *const *sig, int rank, int world,
                             size_t slot_floats, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* FGM_CUDA_H */
