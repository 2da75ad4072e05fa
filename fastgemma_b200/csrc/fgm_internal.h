// Internal launch interfaces between the C ABI (fgm_cuda.cu) and the kernels.
#pragma once

#include <cstddef>
#include <cstdint>
#include <vector>

#include <cuda.h>
#include <cuda_runtime.h>

namespace fgm {

constexpr int kMaxGatherRanks = 8;

// Fused all-gather of a column-sharded decode GEMM (gemv.cu): every rank's
// output buffer has the same [M][ldc] layout; this rank's finished columns
// are also stored into each peer's buffer over NVLink, and system-scope
// counters tell each rank when its buffer is complete.  world = 0: off.
// Which of the two buffers a call uses, and how often that buffer was used
// before, come from the rank's own call counter on the device, so a call's
// launch parameters never change and the call can be replayed from a graph.
struct GatherParams {
  float *out[kMaxGatherRanks];               // each rank's double buffer (slot 0 at out[q])
  unsigned long long *sig[kMaxGatherRanks];  // each rank's signal words (kGatherSigWords x u64)
  size_t slot_floats;                        // floats between slot 0 and slot 1
  int rank, world;
};
// Signal words of one rank (u64 each, zeroed once, never reset):
//   [slot]     ranks whose last CTA finished pushing into this rank's buffer `slot`
//   [2 + slot] ranks that started a call using `slot` (their buffer may be overwritten)
//   [4 + slot] this rank's CTAs done pushing into `slot`
//   [6]        calls this rank completed (slot = calls & 1)
//   [8], [9], [10]  %globaltimer of the last call: CTA 0 start, own pushes done, all arrived
constexpr int kGatherSigWords = 16;

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
  GatherParams g;           // fused all-gather (g.world = 0: none)
  // L2 warm-up of the weights the NEXT launch will stream (up to two regions,
  // 16-byte aligned; bytes 0 = none), prefetched once this launch's own
  // weight stream is queued
  const uint8_t *warm[2];
  size_t warm_bytes[2];
};

// Launch geometry of the streaming decode kernel (gemv.cu).
struct GemvPlan {
  int warps;        // warps per CTA
  int parts;        // warps sharing one n-block (split K), a power of two
  int units;        // n-blocks in the range
  int chunk_tiles;  // weight tiles per ring stage
  int stages;       // ring depth per warp
  int pre_stages;   // ring stages each warp requests before griddepcontrol.wait
  int pub_row;      // words per published row in the split-K exchange area
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
  int8_t *pa;    // may be null (quantised rows only, no tile packing)
  int m, k, hsz, r0, r1;
};

cudaError_t launch_prep(const PrepParams &p, bool pdl, cudaStream_t st);

// ---- decode-chain glue and int8-KV attention (glue.cu)
cudaError_t launch_rmsnorm(float *out, const float *x, const float *w, int rows, int n, float eps,
                           bool pdl, cudaStream_t st);
cudaError_t launch_gelu_mul(float *out, const float *gate, const float *up, int rows, int n,
                            bool pdl, cudaStream_t st);
// op 0: a += b, 1: a *= b, 2: a *= s
cudaError_t launch_elementwise(float *a, const float *b, float s, size_t n, int op, bool pdl,
                               cudaStream_t st);
cudaError_t launch_softcap(float *x, int rows, int n, float cap, bool pdl, cudaStream_t st);
cudaError_t launch_rope(float *x, int x_ld, int rows, int n_heads, int head_dim,
                        const float *inv_freq, const float *tab, int positions, const int *pos,
                        bool pdl, cudaStream_t st);
cudaError_t launch_store_v_t(int8_t *vt, size_t vt_stride, const int8_t *src, int src_ld, int rows,
                             int n, int slot, bool pdl, cudaStream_t st);
struct AttnParams {
  float *out;
  int out_ld;
  const float *q;
  int q_ld;
  const int8_t *kc;       // K [slot][kv_heads * head_dim] per query row
  const float *ks;        // K scales [slot]
  const int8_t *vt;       // V, slot-interleaved (store_v_t)
  const float *vs;        // V scales [slot]
  size_t kc_stride, ks_stride, vt_stride, vs_stride;  // per query row (elements)
  int n_heads, kv_heads, head_dim, start, end, ring;
  int wbase, wslots;      // cache slots [wbase, wbase + wslots) the window can touch
  // set by attend_layout: a cluster of `cluster` CTAs per (row, KV head); CTA
  // c owns the cache slot groups [c*gchunk, +gchunk) above wbase, scores them
  // in stages of kp slots and multiplies them in stages of vg groups; the
  // lane sums gather `win` positions at a time; 16-byte copies when vec16;
  // vgp: V stage storage in groups (vg rounded up to whole 32-slot steps)
  // one: the whole window fits one gather (see the kernel)
  int cluster, gchunk, kp, vg, vgp, win, vec16, one;
  unsigned off_ks, off_k, off_v, off_e, off_win, off_w, off_vsa, off_acc;  // shared memory (bytes)
  size_t smem;
};
// Fused row glue of the decode step (glue.cu).
cudaError_t launch_norm_prep(float *h, const float *proj, const float *w_post, const float *w_pre,
                             int m, int n, float eps, float *qs, int8_t *pa, bool pdl,
                             cudaStream_t st);
cudaError_t launch_gelu_mul_prep(const float *gate, const float *up, int ld, int m, int n,
                                 float *act, float *qs, int8_t *pa, bool pdl, cudaStream_t st);
struct QkvParams {
  float *q, *k, *v;                 // rows q_ld (q) and kv_ld (k, v) floats apart
  int q_ld, kv_ld;
  int n_heads, kv_heads, head_dim;
  const float *q_norm, *k_norm;     // [head_dim]
  float eps;
  const float *inv_freq;            // [head_dim / 2]
  const int *pos;                   // [rows]
  int ring;                         // 0: slot = pos, else pos % ring
  int cap;                          // cache slots per row
  int8_t *kc;
  float *ks;
  int8_t *vt;
  float *vs;
  size_t kc_stride, ks_stride, vt_stride, vs_stride;  // per row (elements)
  const float *rope_tab;            // host-computed cos | sin per position, or null
  int rope_positions;               // positions in rope_tab
};
size_t qkv_post_smem(const QkvParams &p);
cudaError_t launch_qkv_post(const QkvParams &p, int rows, bool pdl, cudaStream_t st);
// Fills the cluster split and the shared memory layout; false when the
// window does not fit in smem_limit bytes.
bool attend_layout(AttnParams &p, size_t smem_limit);
cudaError_t launch_attend_q8(const AttnParams &p, int rows, bool pdl, size_t smem_limit,
                             cudaStream_t st);
// Copy two host regions (device-readable: page-locked or staging) into
// device memory with one kernel.
cudaError_t launch_pull(const void *s1, void *d1, size_t n1, const void *s2, void *d2, size_t n2,
                        bool pdl, cudaStream_t st);

// ----------------------------------------------------------- tensor cores
struct TcParams {
  int M, N, K;
  const int8_t *A;        // row-major int8 activations
  const float *a_scale;
  const float *b_scale;   // int8 per-channel scales [N]
  float *C;
  int ldc, c_col0;
  int32_t *acc;           // raw accumulators [M][N] instead of C (debug launches)
  int nb0;                // first n-block
  int n_end;              // one past the last output column
  int stages;             // ring depth (set by the launcher)
  int *err;
  int tma_store;          // write C through TMA stores (set by the launcher)
  int splits;             // K split across a cluster of this many CTAs (set by the launcher)
  int out_v4;             // C rows 16-byte aligned: vector stores allowed (set by the launcher)
  int m_fast;             // grid x walks the M tiles, y the N tiles (set by the launcher)
};

}  // namespace fgm
#include <cuda.h>
namespace fgm {

// Row-major [rows][ld] byte matrix as a 2-D TMA view, boxes of box_rows x 128
// bytes with the 128-byte swizzle.
bool encode_rows_map(CUtensorMap *map, const void *base, int rows, int K, int ld, int box_rows);
// Tile-packed activations of one 16-row block as a 3-D TMA view, box of
// `rows` rows x K/64 tiles, 64-byte swizzle (K <= 16384).
bool encode_packed_a_map(CUtensorMap *map, const void *base, int K, int rows);
// int4 group scales f16 [groups][N] as a 2-D TMA view, box 16 columns x rows.
bool encode_scale_map(CUtensorMap *map, const void *base, int groups, int N, int rows);
// .fgm int8 tiles -> row-major [N][K] (the tensor-core weight operand).
cudaError_t launch_q8c_rows(const int8_t *tiles, int8_t *rows, int N, int K, cudaStream_t st);
// tile-packed activations -> row-major [M][K].
cudaError_t launch_packed_to_rows(const int8_t *packed, int8_t *rows, int M, int K,
                                  cudaStream_t st);
// p.A is row-major with leading dimension lda bytes.  The launcher picks the
// tile height, K split (cluster size) and ring depth for the device.
cudaError_t launch_q8c_tc(const TcParams &p, int lda, const CUtensorMap &tmB, bool pdl,
                          int num_sms, size_t smem_limit, cudaStream_t st);
constexpr int kTcBoxRowsB = 128;  // output columns per CTA tile

// Row argmax (argmax.cu): partials over column chunks, then merges.
constexpr int kArgmaxChunk = 8192;
int argmax_chunk_count(int N);
cudaError_t launch_argmax_partials(const float *C, int M, int N, int ldc, int col0, float *pv,
                                   int *pi, bool pdl, cudaStream_t st);
cudaError_t launch_argmax_merge(const float *pv, const int *pi, int M, int P, int *out, bool pdl,
                                cudaStream_t st);

// ------------------------------------------------------- decode work list
// worklist.cu: many decode GEMMs and activation preps in one persistent
// launch.  kind: kWlQ4 (int4 q4g GEMM), kWlQ8 (int8 q8c GEMM), kWlPrep (rows
// of fgm_prep_rows into the packed layout).
constexpr int kWlQ4 = 0, kWlQ8 = 1, kWlPrep = 2;
struct WlItem {
  CUtensorMap amap;        // GEMM: packed activations (encode_packed_a_map)
  CUtensorMap smap;        // int4 GEMM: the group scales (encode_scale_map)
  int kind, N, K, gk;      // gk: int4 scale group in 64-value tiles
  int nb0, units;          // GEMM: first n-block and n-blocks; prep: rows (16 per block)
  int ldc, c_col0;         // GEMM: C[m*ldc + n - c_col0]
  int lda, hsz;            // prep: source row stride (floats), FWHT block
  int deps[2];             // earlier items whose outputs this one reads (-1: none)
  int waited;              // some item of the list waits for this one (publish its completion)
  const uint8_t *B;        // GEMM weight tiles
  const void *b_scale;     // f16 [K/group][N] (int4) or f32 [N] (int8)
  const float *a_scale;    // GEMM: [M]
  float *C;
  const float *src;        // prep: f32 rows
  int8_t *pa;              // prep: packed rows
  float *qs;               // prep: row scales
};
constexpr int kWlMaxWarps = 15;  // consumer warps per CTA, at most (16 warps with the producer)
struct WlSeg {                 // one CTA's share of one item
  int item, kind, nst;         // item, its kind, 4 KB weight stages per unit
  int ub, nu;                  // its units: [ub, ub + nu) of the item (n-blocks or rows)
  int gseq;                    // GEMM segments of the CTA before this one (activation slot)
  // the item's fields a unit needs, copied here so one descriptor read
  // serves a unit (no dependent lookup of the item)
  int nb_base;                 // n-block of unit ub
  int ldc, c_col0, gk, waited;
  int ubytes, rows_st;         // weight bytes per unit, int4 scale rows per stage
  float *C;
  const void *b_scale;
  const uint8_t *B;
  const CUtensorMap *smap;     // device address of the item's scale view
};
// One row of a dependency-free prep, prepared at the start of a run by the
// CTA it is dealt to (built on the host: one load fetches it).
struct WlCoopRow {
  const float *src;   // the row's f32 values
  int8_t *pa_row;     // its row of the packed tile block
  float *qs;          // its scale
  int item, hsz;      // the prep entry, its FWHT block
  unsigned pub;       // units it publishes (row 0 also counts the padding rows)
  int nch;            // 128-value chunks
};
constexpr int kWlCoopRows = 16;  // rows a CTA may hold

struct WlParams {
  const WlItem *items;
  int n_items;
  const WlSeg *segs;       // every CTA's segments, back to back
  const int *seg_off;      // CTA c: segs[seg_off[c], seg_off[c + 1])
  unsigned *done;          // per item: units completed in this launch
  unsigned *ctas_done;     // CTAs finished (the last one resets the counters)
  int *abort;              // raised by a warp that gave up on a bounded wait
  int *err;                // device status word
  int M, warps, stages;    // consumer warps per CTA, weight ring stages per warp
  int a_ring;              // bytes of the activation ring (segments staged FIFO)
  const WlCoopRow *coop;   // CTA c's dependency-free prep rows: coop[c*kWlCoopRows + k],
  const int *coop_n;       // k < coop_n[c], prepared at the start of the run
};
struct WlPlan {
  int M, MT, grid, warps, stages, a_ring;
  size_t smem;
  std::vector<WlSeg> segs;
  std::vector<int> seg_off;
  std::vector<WlCoopRow> coop;  // [grid][kWlCoopRows]
  std::vector<int> coop_n;
};
// Fills the schedule and launch geometry; returns an error text or nullptr.
const char *worklist_plan(WlPlan &pl, std::vector<WlItem> &items, int M, int num_sms,
                          size_t smem_optin);
cudaError_t launch_worklist(const WlParams &p, const WlPlan &pl, bool pdl, cudaStream_t st);

// Number of kernel launches issued by this library (instrumentation).
void count_launch(int n = 1);

}  // namespace fgm
