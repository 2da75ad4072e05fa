/*
 * cpu_pool.c -- persistent host thread pool that drives a CPU GEMM kernel the
 * way fastgemma's worker pool does.
 *
 * TEST / BASELINE INFRASTRUCTURE ONLY.  bench.py uses it to time the
 * reference's own CPU kernels (oracle/_ref, AMX or VNNI) or, where those could
 * not be built, the scalar restatement in fgm_oracle.c.  The shipped CUDA
 * library never links it.
 *
 * Behaviour restated from crates/fgm-core/src/pool.rs:
 *  - workers are created once and parked on a start/done barrier pair
 *    (pool.rs:94-99, :244-268); each calls a per-thread init on entry, which
 *    is where AMX tile permission is requested (pool.rs:242);
 *  - a GEMM splits its N/16 n-blocks evenly in whole groups of 4 n-blocks
 *    (split_n / split_gemm, pool.rs:110-124), thread 0 doing the first slice;
 *  - prep splits ceil(M/16) row-tile blocks evenly, and runs on the calling
 *    thread alone below two blocks per thread (Pool::prep, pool.rs:299-311).
 */
#define _GNU_SOURCE
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

typedef void (*q4g_fn)(int, int, int, const int8_t *, const float *,
                       const uint8_t *, const uint16_t *, int, float *, int, int,
                       int);
typedef void (*q8c_fn)(int, int, int, const int8_t *, const float *,
                       const int8_t *, const float *, float *, int, int, int);
typedef void (*prep_fn)(const float *, int, float *, int8_t *, float *, int8_t *,
                        int, int, int, int, int);
typedef int (*init_fn)(void);

enum { JOB_Q4G = 1, JOB_Q8C = 2, JOB_PREP = 3 };

typedef struct {
  int kind;
  void *fn;
  int M, N, K, group, ldc, hsz, lda;
  const void *A, *as, *B, *bs, *src;
  float *C, *rot, *qs;
  int8_t *qa, *pa;
} job_t;

static job_t g_job;
static int g_nt = 0;
static pthread_t *g_th = NULL;
static pthread_barrier_t g_start, g_done;
static volatile int g_stop = 0;
static init_fn g_init = NULL;

/* pool.rs:110-116 */
static void split_n(int total, int nt, int tid, int *a, int *b) {
  int per = total / nt, extra = total % nt;
  int start = tid * per + (tid < extra ? tid : extra);
  *a = start;
  *b = start + per + (tid < extra ? 1 : 0);
}

static void run_slice(const job_t *j, int tid) {
  if (j->kind == JOB_Q4G || j->kind == JOB_Q8C) {
    int a, b;
    split_n(j->N / 16 / 4, g_nt, tid, &a, &b); /* pool.rs:121-124 */
    int n0 = a * 4, n1 = b * 4;
    if (n0 >= n1) return;
    if (j->kind == JOB_Q4G)
      ((q4g_fn)j->fn)(j->M, j->N, j->K, (const int8_t *)j->A, (const float *)j->as,
                      (const uint8_t *)j->B, (const uint16_t *)j->bs, j->group,
                      j->C, j->ldc, n0, n1);
    else
      ((q8c_fn)j->fn)(j->M, j->N, j->K, (const int8_t *)j->A, (const float *)j->as,
                      (const int8_t *)j->B, (const float *)j->bs, j->C, j->ldc,
                      n0, n1);
  } else if (j->kind == JOB_PREP) {
    int blocks = (j->M + 15) / 16, b0, b1;
    split_n(blocks, g_nt, tid, &b0, &b1);
    int r0 = b0 * 16, r1 = b1 * 16 < j->M ? b1 * 16 : j->M; /* pool.rs:206-225 */
    if (r0 >= r1) return;
    ((prep_fn)j->fn)((const float *)j->src, j->lda, j->rot, j->qa, j->qs, j->pa,
                     j->M, j->K, j->hsz, r0, r1);
  }
}

static void *worker(void *arg) {
  int tid = (int)(intptr_t)arg;
  if (g_init) g_init();
  for (;;) {
    pthread_barrier_wait(&g_start);
    if (g_stop) return NULL;
    run_slice(&g_job, tid);
    pthread_barrier_wait(&g_done);
  }
}

/* Start nt threads in total (the caller counts as thread 0).  `init` runs once
 * on every thread, the caller included, before any work. */
int cpu_pool_start(int nt, init_fn init) {
  if (g_nt) return -1;
  if (nt < 1) nt = 1;
  g_nt = nt;
  g_init = init;
  g_stop = 0;
  if (init) init();
  if (nt == 1) return 0;
  pthread_barrier_init(&g_start, NULL, nt);
  pthread_barrier_init(&g_done, NULL, nt);
  g_th = calloc((size_t)nt, sizeof(pthread_t));
  for (int t = 1; t < nt; t++)
    pthread_create(&g_th[t], NULL, worker, (void *)(intptr_t)t);
  return 0;
}

void cpu_pool_stop(void) {
  if (!g_nt) return;
  if (g_nt > 1) {
    g_stop = 1;
    pthread_barrier_wait(&g_start);
    for (int t = 1; t < g_nt; t++) pthread_join(g_th[t], NULL);
    pthread_barrier_destroy(&g_start);
    pthread_barrier_destroy(&g_done);
    free(g_th);
    g_th = NULL;
  }
  g_nt = 0;
}

int cpu_pool_threads(void) { return g_nt; }

static void dispatch(int parallel) {
  if (g_nt == 1 || !parallel) {
    int saved = g_nt;
    g_nt = 1;
    run_slice(&g_job, 0);
    g_nt = saved;
    return;
  }
  pthread_barrier_wait(&g_start);
  run_slice(&g_job, 0);
  pthread_barrier_wait(&g_done);
}

/* Pool::gemm (pool.rs:285-295) for an int4 kernel with the fgm_gemm_q4g ABI. */
void cpu_pool_gemm_q4g(q4g_fn fn, int M, int N, int K, const int8_t *A,
                       const float *as, const uint8_t *Bq, const uint16_t *bs,
                       int group, float *C, int ldc) {
  job_t j = {0};
  j.kind = JOB_Q4G; j.fn = (void *)fn; j.M = M; j.N = N; j.K = K; j.A = A;
  j.as = as; j.B = Bq; j.bs = bs; j.group = group; j.C = C; j.ldc = ldc;
  g_job = j;
  dispatch(1);
}

/* Pool::gemm for an int8 kernel with the fgm_gemm_q8c ABI. */
void cpu_pool_gemm_q8c(q8c_fn fn, int M, int N, int K, const int8_t *A,
                       const float *as, const int8_t *B, const float *bs,
                       float *C, int ldc) {
  job_t j = {0};
  j.kind = JOB_Q8C; j.fn = (void *)fn; j.M = M; j.N = N; j.K = K; j.A = A;
  j.as = as; j.B = B; j.bs = bs; j.C = C; j.ldc = ldc;
  g_job = j;
  dispatch(1);
}

/* Pool::prep (pool.rs:299-311) for a kernel with the fgm_prep_rows ABI. */
void cpu_pool_prep(prep_fn fn, const float *src, int lda, float *rot, int8_t *qa,
                   float *qs, int8_t *pa, int m, int k, int hsz) {
  job_t j = {0};
  j.kind = JOB_PREP; j.fn = (void *)fn; j.src = src; j.lda = lda; j.rot = rot;
  j.qa = qa; j.qs = qs; j.pa = pa; j.M = m; j.K = k; j.hsz = hsz;
  g_job = j;
  int blocks = (m + 15) / 16;
  dispatch(!(g_nt == 1 || blocks < g_nt * 2));
}

double cpu_pool_now(void) {
  struct timespec t;
  clock_gettime(CLOCK_MONOTONIC, &t);
  return (double)t.tv_sec + 1e-9 * (double)t.tv_nsec;
}
