// C ABI of the sm_100a backend (include/fgm_cuda.h): argument contracts,
// device selection, the weight registry, host-pointer drop-ins and the
// device-pointer entry points.

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "fgm_cuda.h"
#include "fgm_internal.h"

namespace fgm {

static std::atomic<uint64_t> g_launches{0};
void count_launch(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }

static thread_local std::string t_err;

// Bumped whenever a device address a cached call graph may hold can change
// (registry, staging growth, prepared weights); see host_linear.
static std::atomic<uint64_t> g_gen{1};
static void bump_gen() { g_gen.fetch_add(1, std::memory_order_relaxed); }

static int fail(int code, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_err = buf;
  return code;
}

static int cuda_fail(cudaError_t e, const char *what) {
  return fail(FGM_CUDA_ERUNTIME, "%s: %s", what, cudaGetErrorString(e));
}

#define FGM_TRY(call)                                            \
  do {                                                           \
    cudaError_t e_ = (call);                                     \
    if (e_ != cudaSuccess) return cuda_fail(e_, #call);          \
  } while (0)

// ------------------------------------------------------------------ contracts
static int check_gemm(int M, int N, int K, int ldc, int n0, int n1, int group, bool q4) {
  if (M < 0) return fail(FGM_CUDA_EINVAL, "M=%d < 0", M);
  if (K <= 0 || K % 64 != 0 || K > 65536)
    return fail(FGM_CUDA_EINVAL, "K=%d: need 0 < K <= 65536 and K %% 64 == 0", K);
  if (N <= 0 || N % 16 != 0) return fail(FGM_CUDA_EINVAL, "N=%d: need N > 0 and N %% 16 == 0", N);
  if (n0 < 0 || n1 < n0 || n1 > N / 16)
    return fail(FGM_CUDA_EINVAL, "n-block range [%d, %d) outside [0, %d]", n0, n1, N / 16);
  if ((n1 - n0) % 4 != 0)
    return fail(FGM_CUDA_EINVAL, "n-block range [%d, %d) is not a multiple of 4", n0, n1);
  if (ldc < N) return fail(FGM_CUDA_EINVAL, "ldc=%d < N=%d", ldc, N);
  if (q4 && (group <= 0 || group % 64 != 0 || K % group != 0))
    return fail(FGM_CUDA_EINVAL, "group=%d: need group > 0, group %% 64 == 0, K %% group == 0",
                group);
  return FGM_CUDA_OK;
}

static int check_prep(int lda, int m, int k, int hsz, int r0, int r1, bool have_qa) {
  if (m < 0) return fail(FGM_CUDA_EINVAL, "m=%d < 0", m);
  if (k <= 0 || k % 64 != 0 || k > 65536)
    return fail(FGM_CUDA_EINVAL, "k=%d: need 0 < k <= 65536 and k %% 64 == 0", k);
  if (lda < k) return fail(FGM_CUDA_EINVAL, "lda=%d < k=%d", lda, k);
  if (hsz < 0 || (hsz > 0 && ((hsz & (hsz - 1)) != 0 || k % hsz != 0)))
    return fail(FGM_CUDA_EINVAL, "hsz=%d: need 0 or a power of two dividing k=%d", hsz, k);
  if (r0 < 0 || r0 % 16 != 0 || r1 > m || (r1 < r0))
    return fail(FGM_CUDA_EINVAL, "rows [%d, %d) of m=%d: need r0 %% 16 == 0, r0 <= r1 <= m", r0,
                r1, m);
  if (r1 < m && r1 % 16 != 0 && !have_qa)
    return fail(FGM_CUDA_EINVAL, "a row range ending inside a tile block needs qa");
  return FGM_CUDA_OK;
}

static size_t packed_len(int m, int k) { return (size_t)((m + 15) / 16) * 16 * (size_t)k; }

// ------------------------------------------------------------------- device
static std::mutex g_dev_mu;
static int g_dev = -1;
static cudaStream_t g_stream = nullptr;

static int pick_device(int want) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
    cudaGetLastError();
    return fail(FGM_CUDA_ENODEV, "no CUDA device visible");
  }
  int dev = want;
  if (dev < 0) {
    const char *e = getenv("FGM_CUDA_DEVICE");
    if (e && *e) dev = atoi(e);
    else if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
  }
  if (dev < 0 || dev >= n) return fail(FGM_CUDA_ENODEV, "device %d of %d", dev, n);
  cudaDeviceProp prop;
  FGM_TRY(cudaGetDeviceProperties(&prop, dev));
  if (prop.major != 10)
    return fail(FGM_CUDA_ENODEV, "device %d is sm_%d%d; this build targets sm_100a", dev,
                prop.major, prop.minor);
  return dev;
}

static int ensure_device() {
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (g_dev < 0) {
    int dev = pick_device(-1);
    if (dev < 0) return dev;
    FGM_TRY(cudaSetDevice(dev));
    FGM_TRY(cudaStreamCreateWithFlags(&g_stream, cudaStreamNonBlocking));
    g_dev = dev;
  } else {
    FGM_TRY(cudaSetDevice(g_dev));
  }
  return FGM_CUDA_OK;
}

// ----------------------------------------------------------------- registry
struct RegEntry {
  void *dev;
  size_t bytes;
};
static std::mutex g_reg_mu;
static std::unordered_map<const void *, RegEntry> g_reg;
static size_t g_reg_bytes = 0;

static int reg_upload(const void *host, size_t bytes, const void **dev) {
  std::lock_guard<std::mutex> lk(g_reg_mu);
  auto it = g_reg.find(host);
  if (it != g_reg.end()) {
    if (it->second.bytes != bytes)
      return fail(FGM_CUDA_EINVAL, "weight %p registered with %zu bytes, now %zu", host,
                  it->second.bytes, bytes);
    *dev = it->second.dev;
    return FGM_CUDA_OK;
  }
  void *d = nullptr;
  if (cudaMalloc(&d, bytes) != cudaSuccess) {
    cudaGetLastError();
    return fail(FGM_CUDA_ENOMEM, "cudaMalloc(%zu) for weight %p", bytes, host);
  }
  cudaError_t e = cudaMemcpy(d, host, bytes, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(d);
    return cuda_fail(e, "weight upload");
  }
  g_reg[host] = RegEntry{d, bytes};
  g_reg_bytes += bytes;
  bump_gen();
  *dev = d;
  return FGM_CUDA_OK;
}

// Device copy of a registered blob, or nullptr.  A registered blob must span
// at least `bytes`; an unregistered one is the caller's to upload per call.
static int reg_find(const void *host, size_t bytes, const void **dev) {
  std::lock_guard<std::mutex> lk(g_reg_mu);
  auto it = g_reg.find(host);
  *dev = nullptr;
  if (it == g_reg.end()) return FGM_CUDA_OK;
  if (it->second.bytes < bytes)
    return fail(FGM_CUDA_EINVAL, "weight %p registered with %zu bytes, call needs %zu", host,
                it->second.bytes, bytes);
  *dev = it->second.dev;
  return FGM_CUDA_OK;
}

// ------------------------------------------------------------ host staging
// One pinned host buffer and one device buffer, grown geometrically and kept:
// after the first call of a given size the host path allocates nothing.
struct Staging {
  char *h = nullptr;
  size_t hcap = 0;
  char *d = nullptr;
  size_t dcap = 0;
};
static std::mutex g_host_mu;  // serialises the host-pointer entry points
static Staging g_stage;

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

static int stage_reserve(size_t bytes) {
  if (bytes > g_stage.hcap) {
    size_t cap = std::max(bytes, g_stage.hcap * 2);
    if (g_stage.h) cudaFreeHost(g_stage.h);
    g_stage.h = nullptr;
    g_stage.hcap = 0;
    if (cudaMallocHost(&g_stage.h, cap) != cudaSuccess) {
      cudaGetLastError();
      return fail(FGM_CUDA_ENOMEM, "cudaMallocHost(%zu)", cap);
    }
    g_stage.hcap = cap;
    bump_gen();
  }
  if (bytes > g_stage.dcap) {
    size_t cap = std::max(bytes, g_stage.dcap * 2);
    if (g_stage.d) cudaFree(g_stage.d);
    g_stage.d = nullptr;
    g_stage.dcap = 0;
    if (cudaMalloc(&g_stage.d, cap) != cudaSuccess) {
      cudaGetLastError();
      return fail(FGM_CUDA_ENOMEM, "cudaMalloc(%zu)", cap);
    }
    g_stage.dcap = cap;
    bump_gen();
  }
  return FGM_CUDA_OK;
}

static bool is_pinned(const void *p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeHost;
}

// Copy `bytes` from host `src` to device `dst` (through staging at `hoff`
// unless src is pinned).
static int h2d(void *dst, const void *src, size_t bytes, size_t hoff) {
  if (!bytes) return FGM_CUDA_OK;
  if (is_pinned(src)) {
    FGM_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, g_stream));
  } else {
    memcpy(g_stage.h + hoff, src, bytes);
    FGM_TRY(cudaMemcpyAsync(dst, g_stage.h + hoff, bytes, cudaMemcpyHostToDevice, g_stream));
  }
  return FGM_CUDA_OK;
}

// A device-readable address for `bytes` of host data: page-locked memory is
// read in place over PCIe (unified addressing, no copy); pageable memory is
// copied into the pinned staging buffer at `hoff` (a host memcpy, no DMA).
// The caller keeps the data untouched until its work has completed (the
// host-pointer entry points synchronise before returning).
static int host_readable(const void *src, size_t bytes, size_t hoff, const void **dev) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, src) == cudaSuccess && a.type == cudaMemoryTypeHost &&
      a.devicePointer) {
    *dev = a.devicePointer;
    return FGM_CUDA_OK;
  }
  cudaGetLastError();
  memcpy(g_stage.h + hoff, src, bytes);
  void *dp = nullptr;
  FGM_TRY(cudaHostGetDevicePointer(&dp, g_stage.h + hoff, 0));
  *dev = dp;
  return FGM_CUDA_OK;
}

// Copy-back of rows [0, rows) x `width` bytes of a compact device matrix to
// host memory with pitch `hpitch`: enqueue (straight into page-locked
// memory, else into staging at `hoff`), then finish (wait, and move staged
// rows into place).
static int d2h_rows_enqueue(void *dst, size_t hpitch, const void *dsrc, size_t width, int rows,
                            size_t hoff, bool pinned) {
  if (rows <= 0 || width == 0) return FGM_CUDA_OK;
  if (pinned)
    FGM_TRY(cudaMemcpy2DAsync(dst, hpitch, dsrc, width, width, rows, cudaMemcpyDeviceToHost,
                              g_stream));
  else
    FGM_TRY(cudaMemcpyAsync(g_stage.h + hoff, dsrc, width * rows, cudaMemcpyDeviceToHost,
                            g_stream));
  return FGM_CUDA_OK;
}

static int d2h_rows_finish(void *dst, size_t hpitch, size_t width, int rows, size_t hoff,
                           bool pinned) {
  FGM_TRY(cudaStreamSynchronize(g_stream));
  if (!pinned)
    for (int r = 0; r < rows; r++)
      memcpy((char *)dst + (size_t)r * hpitch, g_stage.h + hoff + (size_t)r * width, width);
  return FGM_CUDA_OK;
}

// Rows [0, rows) x `width` bytes of a compact device matrix into host memory
// with pitch `hpitch`, then wait.
static int d2h_rows_sync(void *dst, size_t hpitch, const void *dsrc, size_t width, int rows,
                         size_t hoff) {
  if (rows <= 0 || width == 0) {
    FGM_TRY(cudaStreamSynchronize(g_stream));
    return FGM_CUDA_OK;
  }
  if (is_pinned(dst)) {
    FGM_TRY(cudaMemcpy2DAsync(dst, hpitch, dsrc, width, width, rows, cudaMemcpyDeviceToHost,
                              g_stream));
    FGM_TRY(cudaStreamSynchronize(g_stream));
  } else {
    FGM_TRY(cudaMemcpyAsync(g_stage.h + hoff, dsrc, width * rows, cudaMemcpyDeviceToHost,
                            g_stream));
    FGM_TRY(cudaStreamSynchronize(g_stream));
    for (int r = 0; r < rows; r++)
      memcpy((char *)dst + (size_t)r * hpitch, g_stage.h + hoff + (size_t)r * width, width);
  }
  return FGM_CUDA_OK;
}

// ------------------------------------------------- per-device launch facts
struct DevInfo {
  int sms = 0;
  size_t smem_optin = 0;
  int *err = nullptr;  // bounded-wait failure flag, cleared by fgm_cuda_device_status
};
static std::mutex g_info_mu;
static DevInfo g_info[64];

static int dev_info(DevInfo **out) {
  int dev = 0;
  FGM_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(FGM_CUDA_ENODEV, "device index %d", dev);
  std::lock_guard<std::mutex> lk(g_info_mu);
  DevInfo &d = g_info[dev];
  if (!d.sms) {
    int v = 0;
    FGM_TRY(cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev));
    int sm = 0;
    FGM_TRY(cudaDeviceGetAttribute(&sm, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    void *e = nullptr;
    FGM_TRY(cudaMalloc(&e, 256));
    FGM_TRY(cudaMemset(e, 0, 256));
    d.err = static_cast<int *>(e);
    d.smem_optin = (size_t)sm - 1024;  // headroom for the kernels' static shared memory
    d.sms = v;
  }
  *out = &d;
  return FGM_CUDA_OK;
}

// PDL (programmatic dependent launch) lets a kernel's weight prefetch overlap
// the tail of the kernel before it.  FGM_CUDA_PDL=0 turns it off.
static bool use_pdl() {
  static int v = -1;
  if (v < 0) {
    const char *e = getenv("FGM_CUDA_PDL");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

static bool aligned16(const void *p) { return ((uintptr_t)p & 15u) == 0; }

// --------------------------------------------- prepared tensor-core operands
// int8 weights as the row-major [N][K] operand the tcgen05 kernel reads, keyed
// by the device address of the .fgm copy they were made from.
struct Prepared {
  int8_t *kmajor;
  size_t bytes;
  int N, K;
  CUtensorMap map;
};
static std::mutex g_prep_mu;
static std::unordered_map<const void *, Prepared> g_prep;

static int tc_min_m() {
  static int v = -1;
  if (v < 0) {
    const char *e = getenv("FGM_CUDA_TC_MIN_M");
    v = (e && *e) ? atoi(e) : 64;
  }
  return v;
}

static int prepare_q8c(const int8_t *B, int N, int K, cudaStream_t st) {
  std::lock_guard<std::mutex> lk(g_prep_mu);
  auto it = g_prep.find(B);
  if (it != g_prep.end()) {
    if (it->second.N != N || it->second.K != K)
      return fail(FGM_CUDA_EINVAL, "weight %p prepared as %dx%d, now %dx%d", (const void *)B,
                  it->second.N, it->second.K, N, K);
    return FGM_CUDA_OK;
  }
  Prepared pr{};
  pr.bytes = (size_t)N * K;
  pr.N = N;
  pr.K = K;
  if (cudaMalloc(&pr.kmajor, pr.bytes) != cudaSuccess) {
    cudaGetLastError();
    return fail(FGM_CUDA_ENOMEM, "cudaMalloc(%zu) for a prepared weight", pr.bytes);
  }
  cudaError_t e = launch_q8c_rows(B, pr.kmajor, N, K, st);
  if (e != cudaSuccess) {
    cudaFree(pr.kmajor);
    return cuda_fail(e, "q8c repack");
  }
  count_launch();
  if (!encode_rows_map(&pr.map, pr.kmajor, N, K, K, kTcBoxRowsB)) {
    cudaFree(pr.kmajor);
    return fail(FGM_CUDA_ERUNTIME, "cuTensorMapEncodeTiled failed for a prepared weight");
  }
  g_prep[B] = pr;
  bump_gen();
  return FGM_CUDA_OK;
}

static bool find_prepared(const void *B, CUtensorMap *map) {
  std::lock_guard<std::mutex> lk(g_prep_mu);
  auto it = g_prep.find(B);
  if (it == g_prep.end()) return false;
  *map = it->second.map;
  return true;
}

static void release_prepared(const void *B) {
  std::lock_guard<std::mutex> lk(g_prep_mu);
  auto it = g_prep.find(B);
  if (it == g_prep.end()) return;
  cudaFree(it->second.kmajor);
  g_prep.erase(it);
  bump_gen();
}

// A is row-major [M][lda] int8.
static int run_q8c_tc(int M, int N, int K, const int8_t *A, int lda, const float *a_scale,
                      const float *b_scale, const CUtensorMap &map, float *C, int ldc, int c_col0,
                      int32_t *acc, int n0, int n1, cudaStream_t st) {
  DevInfo *di = nullptr;
  int rc = dev_info(&di);
  if (rc) return rc;
  if (!aligned16(A) || lda % 16 != 0)
    return fail(FGM_CUDA_EINVAL, "row-major activations need 16-byte aligned rows");
  if (b_scale && !aligned16(b_scale))
    return fail(FGM_CUDA_EINVAL, "int8 weight scales must be 16-byte aligned");
  TcParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.A = A;
  p.a_scale = a_scale;
  p.b_scale = b_scale;
  p.C = C;
  p.ldc = ldc;
  p.c_col0 = c_col0;
  p.acc = acc;
  p.nb0 = n0;
  p.n_end = n1 * 16;
  p.err = di->err;
  cudaError_t e = launch_q8c_tc(p, lda, map, use_pdl(), di->sms, di->smem_optin, st);
  if (e != cudaSuccess) return cuda_fail(e, "gemm_q8c tensor-core launch");
  count_launch();
  return FGM_CUDA_OK;
}

// Tile-packed A on the tensor-core path: a row-major copy in stream-ordered
// temporary memory (so concurrent streams never share it), then the GEMM.
static int run_q8c_tc_packed(int M, int N, int K, const int8_t *A, const float *a_scale,
                             const float *b_scale, const CUtensorMap &map, float *C, int ldc,
                             int c_col0, int32_t *acc, int n0, int n1, cudaStream_t st) {
  void *rows = nullptr;
  FGM_TRY(cudaMallocAsync(&rows, (size_t)M * K, st));
  cudaError_t e = launch_packed_to_rows(A, static_cast<int8_t *>(rows), M, K, st);
  int rc = FGM_CUDA_OK;
  if (e != cudaSuccess) rc = cuda_fail(e, "activation repack");
  else {
    count_launch();
    rc = run_q8c_tc(M, N, K, static_cast<int8_t *>(rows), K, a_scale, b_scale, map, C, ldc,
                    c_col0, acc, n0, n1, st);
  }
  cudaError_t f = cudaFreeAsync(rows, st);
  if (!rc && f != cudaSuccess) rc = cuda_fail(f, "cudaFreeAsync");
  return rc;
}

// ------------------------------- tensor-core path without device allocation
// Some callers must not allocate device memory once they are serving: an
// engine that reserves its whole HBM budget for weights and the KV cache at
// start-up (a stream-ordered allocation can then fail with out-of-memory in
// the middle of a request), and host-language callers that reach this library
// only through the C ABI and hold no say over the process's CUDA memory pools.
// For them fgm_cuda_gemm_q8c_noalloc keeps the row-major activation copy in
// this fixed file-scope buffer instead of stream-ordered temporary memory.
// Every call on a device shares the one buffer, so calls that overlap in time
// (different streams or host threads) race on it; calls on one stream are
// ordered and safe.  Nothing in it has to start at zero: the repack writes
// all M*K bytes before the GEMM reads them, and the rows past M of the last
// 256-row tile come from the TMA zero fill of the M-row activation view.
constexpr size_t kStaticRowsBytes = (size_t)4 << 20;  // M*K limit (e.g. 256 x 16384)
static __device__ __align__(256) int8_t g_static_rows[kStaticRowsBytes];

static std::mutex g_static_mu;
static int8_t *g_static_ptr[64];

// The buffer's address on the current device, looked up once per device.
// The first lookup can load the module, so it is set-up work: make the first
// call on each device before any stream capture.
static int static_rows(int8_t **out) {
  int dev = 0;
  FGM_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(FGM_CUDA_ENODEV, "device index %d", dev);
  std::lock_guard<std::mutex> lk(g_static_mu);
  if (!g_static_ptr[dev]) {
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_static_rows);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(static activation rows)");
    g_static_ptr[dev] = static_cast<int8_t *>(p);
  }
  *out = g_static_ptr[dev];
  return FGM_CUDA_OK;
}

// ------------------------------------------------------------- launchers
struct Warm {
  const void *p[2] = {nullptr, nullptr};
  size_t bytes[2] = {0, 0};
};

static int run_gemm(bool q4, int M, int N, int K, const int8_t *A, const float *a_scale,
                    const void *B, const void *b_scale, int group, float *C, int ldc, int c_col0,
                    int32_t *acc, int n0, int n1, cudaStream_t st, const Warm &warm = Warm()) {
  if (M == 0 || n0 == n1) return FGM_CUDA_OK;
  if (!aligned16(B) || (q4 && b_scale && !aligned16(b_scale)))
    return fail(FGM_CUDA_EINVAL, "weights and int4 scales must be 16-byte aligned");
  CUtensorMap map;
  if (!q4 && M >= tc_min_m() && find_prepared(B, &map))
    return run_q8c_tc_packed(M, N, K, A, a_scale, static_cast<const float *>(b_scale), map, C,
                             ldc, c_col0, acc, n0, n1, st);
  DevInfo *di = nullptr;
  int rc = dev_info(&di);
  if (rc) return rc;
  GemvParams p{};
  p.err = di->err;
  p.M = M;
  p.N = N;
  p.K = K;
  p.group = q4 ? group : 0;
  p.A = A;
  p.a_scale = a_scale;
  p.B = static_cast<const uint8_t *>(B);
  p.b_scale = b_scale;
  p.C = C;
  p.ldc = ldc;
  p.c_col0 = c_col0;
  p.acc = acc;
  p.nb0 = n0;
  for (int r = 0; r < 2; r++) {
    p.warm[r] = static_cast<const uint8_t *>(warm.p[r]);
    p.warm_bytes[r] = warm.p[r] ? warm.bytes[r] : 0;
  }
  cudaError_t e = launch_gemv(p, n1 - n0, q4, use_pdl(), di->sms, di->smem_optin, st);
  if (e != cudaSuccess) return cuda_fail(e, q4 ? "gemm_q4g launch" : "gemm_q8c launch");
  count_launch();
  return FGM_CUDA_OK;
}

static int run_prep(const float *src, int lda, float *rot, int8_t *qa, float *qs, int8_t *pa,
                    int m, int k, int hsz, int r0, int r1, cudaStream_t st) {
  if (r0 >= r1) return FGM_CUDA_OK;
  PrepParams p{src, lda, rot, qa, qs, pa, m, k, hsz, r0, r1};
  cudaError_t e = launch_prep(p, use_pdl(), st);
  if (e != cudaSuccess) return cuda_fail(e, "prep launch");
  count_launch();
  return FGM_CUDA_OK;
}

// ------------------------------------------------------------- Gemm::run
// One projection of fgm-core's Gemm::run (forward.rs:128-158) on device
// buffers: the prep kernel writes the packed (and, for the tensor cores,
// row-major) int8 rows to stream-ordered temporary memory, then the GEMM.
static int run_linear(bool q4, const float *src, int lda, int hsz, int M, int N, int K,
                      const void *B, const void *b_scale, int group, float *C, int ldc, int n0,
                      int n1, cudaStream_t st) {
  if (M == 0 || n0 == n1) return FGM_CUDA_OK;
  CUtensorMap map;
  const bool tc = !q4 && M >= tc_min_m() && find_prepared(B, &map);
  const size_t a_len = packed_len(M, K), o_s = align256(a_len);
  const size_t o_q = o_s + align256((size_t)M * 4), total = o_q + (tc ? align256((size_t)M * K) : 0);
  void *tmp = nullptr;
  FGM_TRY(cudaMallocAsync(&tmp, total, st));
  char *d = static_cast<char *>(tmp);
  int8_t *qa = tc ? reinterpret_cast<int8_t *>(d + o_q) : nullptr;
  float *qs = reinterpret_cast<float *>(d + o_s);
  int rc = run_prep(src, lda, nullptr, qa, qs, reinterpret_cast<int8_t *>(d), M, K, hsz, 0, M, st);
  if (!rc) {
    if (tc)
      rc = run_q8c_tc(M, N, K, qa, K, qs, static_cast<const float *>(b_scale), map, C, ldc, 0,
                      nullptr, n0, n1, st);
    else
      rc = run_gemm(q4, M, N, K, reinterpret_cast<const int8_t *>(d), qs, B, b_scale, group, C,
                    ldc, 0, nullptr, n0, n1, st);
  }
  const cudaError_t f = cudaFreeAsync(tmp, st);
  if (!rc && f != cudaSuccess) rc = cuda_fail(f, "cudaFreeAsync");
  return rc;
}

// Host-pointer GEMM: stage A and a_scale, resolve weights, run, bring back C.
// ----------------------------------------------------- replayed host calls
// A host-pointer call repeating the pointers and shapes of an earlier one
// (the steady state of an inference loop) replays an instantiated CUDA graph
// of its device work -- prep, GEMM, copy-back -- with one launch instead of
// one API call and one queue gap per operation.  The graph is captured on
// the second occurrence (the first one warms every per-shape cache outside
// capture).  Every graph is dropped when g_gen moves.
struct CallKey {
  const void *src, *src2, *B, *bs;  // src2: the activation scales of a gemm call
  void *C;
  int kind;  // 0: linear (prep + GEMM), 1: gemm (pull + GEMM)
  int q4, lda, hsz, M, N, K, group, ldc, n0, n1, src_pinned, c_pinned;
  bool operator==(const CallKey &o) const { return memcmp(this, &o, sizeof(CallKey)) == 0; }
};
struct CallKeyHash {
  size_t operator()(const CallKey &k) const {
    const unsigned char *p = reinterpret_cast<const unsigned char *>(&k);
    size_t h = 1469598103934665603ull;
    for (size_t i = 0; i < sizeof(CallKey); i++) h = (h ^ p[i]) * 1099511628211ull;
    return h;
  }
};
constexpr size_t kMaxCallGraphs = 512;
static std::unordered_map<CallKey, cudaGraphExec_t, CallKeyHash> g_call_graphs;
static std::unordered_map<CallKey, int, CallKeyHash> g_calls_seen;
static uint64_t g_call_graphs_gen = 0;

static void drop_call_graphs() {
  for (auto &kv : g_call_graphs) cudaGraphExecDestroy(kv.second);
  g_call_graphs.clear();
  g_calls_seen.clear();
}

// Run `enqueue` (device work on g_stream) for `key`: replay, capture or plain.
template <class F>
static int run_call(const CallKey &key, F &&enqueue) {
  const uint64_t gen = g_gen.load(std::memory_order_relaxed);
  if (g_call_graphs_gen != gen) {
    drop_call_graphs();
    g_call_graphs_gen = gen;
  }
  auto it = g_call_graphs.find(key);
  if (it != g_call_graphs.end()) {
    FGM_TRY(cudaGraphLaunch(it->second, g_stream));
    return FGM_CUDA_OK;
  }
  if (!g_calls_seen.count(key)) {
    g_calls_seen[key] = 1;
    return enqueue();
  }
  if (g_call_graphs.size() >= kMaxCallGraphs) drop_call_graphs();
  FGM_TRY(cudaStreamBeginCapture(g_stream, cudaStreamCaptureModeThreadLocal));
  const int rc = enqueue();
  cudaGraph_t graph = nullptr;
  const cudaError_t ce = cudaStreamEndCapture(g_stream, &graph);
  if (rc) {
    if (ce == cudaSuccess && graph) cudaGraphDestroy(graph);
    return rc;
  }
  FGM_TRY(ce);
  cudaGraphExec_t exec = nullptr;
  const cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  FGM_TRY(ie);
  g_call_graphs[key] = exec;
  FGM_TRY(cudaGraphLaunch(exec, g_stream));
  return FGM_CUDA_OK;
}

static int host_gemm(bool q4, int M, int N, int K, const int8_t *A, const float *a_scale,
                     const void *B, const void *b_scale, int group, float *C, int ldc, int n0,
                     int n1) {
  int rc = check_gemm(M, N, K, ldc, n0, n1, group, q4);
  if (rc) return rc;
  if (M == 0 || n0 == n1) return FGM_CUDA_OK;
  if (!A || !a_scale || !B || !b_scale || !C) return fail(FGM_CUDA_EINVAL, "null pointer");
  std::lock_guard<std::mutex> lk(g_host_mu);
  if ((rc = ensure_device())) return rc;
  const void *dB = nullptr, *dS = nullptr;
  const size_t wbytes = q4 ? (size_t)N * K / 2 : (size_t)N * K;
  const size_t sbytes = q4 ? (size_t)(K / group) * N * 2 : (size_t)N * 4;
  if ((rc = reg_find(B, wbytes, &dB))) return rc;
  if ((rc = reg_find(b_scale, sbytes, &dS))) return rc;
  const int cols = (n1 - n0) * 16;
  const size_t a_len = packed_len(M, K), s_len = (size_t)M * 4, c_len = (size_t)M * cols * 4;
  const size_t o_s = align256(a_len), o_c = o_s + align256(s_len), o_w = o_c + align256(c_len);
  const size_t o_ws = o_w + (dB ? 0 : align256(wbytes));
  const size_t total = o_ws + (dS ? 0 : align256(sbytes));
  if ((rc = stage_reserve(total))) return rc;
  char *d = g_stage.d;
  // A and a_scale: read through their device mapping when page-locked, else
  // from the pinned staging buffer; one small kernel moves both into device
  // memory (no copy-engine round trips)
  const void *a_src = nullptr, *s_src = nullptr;
  if ((rc = host_readable(A, a_len, 0, &a_src))) return rc;
  if ((rc = host_readable(a_scale, s_len, o_s, &s_src))) return rc;
  if (!dB) {  // unregistered weights: this call's own upload
    if ((rc = h2d(d + o_w, B, wbytes, o_w))) return rc;
    dB = d + o_w;
  } else if (!q4 && M >= tc_min_m()) {  // resident int8 weights: tensor-core operand copy
    if ((rc = prepare_q8c(static_cast<const int8_t *>(dB), N, K, g_stream))) return rc;
  }
  if (!dS) {
    if ((rc = h2d(d + o_ws, b_scale, sbytes, o_ws))) return rc;
    dS = d + o_ws;
  }
  // Page-locked C (decode GEMM): outputs go straight into it through the
  // device mapping, element (m, n) at C[m*ldc + n]; otherwise through the
  // device buffer and one copy.
  const bool c_pinned = is_pinned(C);
  float *c_mapped = nullptr;
  if (!(!q4 && M >= tc_min_m()) && c_pinned) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, C) == cudaSuccess && a.devicePointer)
      c_mapped = static_cast<float *>(a.devicePointer);
    else
      cudaGetLastError();
  }
  auto enqueue = [&]() -> int {
    cudaError_t e = launch_pull(a_src, d, a_len, s_src, d + o_s, s_len, use_pdl(), g_stream);
    if (e != cudaSuccess) return cuda_fail(e, "activation pull launch");
    count_launch();
    int r;
    if (c_mapped)
      r = run_gemm(q4, M, N, K, (const int8_t *)d, (const float *)(d + o_s), dB, dS, group,
                   c_mapped + (size_t)n0 * 16, ldc, n0 * 16, nullptr, n0, n1, g_stream);
    else
      r = run_gemm(q4, M, N, K, (const int8_t *)d, (const float *)(d + o_s), dB, dS, group,
                   (float *)(d + o_c), cols, n0 * 16, nullptr, n0, n1, g_stream);
    if (r || c_mapped) return r;
    return d2h_rows_enqueue(C + (size_t)n0 * 16, (size_t)ldc * 4, d + o_c, (size_t)cols * 4, M,
                            o_c, c_pinned);
  };
  if (dB != d + o_w && dS != d + o_ws) {  // registered weights: every address is stable
    CallKey key;
    memset(&key, 0, sizeof(key));
    key.kind = 1;
    key.src = A;
    key.src2 = a_scale;
    key.B = B;
    key.bs = b_scale;
    key.C = C;
    key.q4 = q4;
    key.M = M;
    key.N = N;
    key.K = K;
    key.group = group;
    key.ldc = ldc;
    key.n0 = n0;
    key.n1 = n1;
    key.src_pinned = (a_src == static_cast<const void *>(A)) | ((s_src == a_scale) << 1);
    key.c_pinned = c_pinned;
    rc = run_call(key, enqueue);
  } else {
    rc = enqueue();
  }
  if (rc) return rc;
  if (c_mapped) {
    FGM_TRY(cudaStreamSynchronize(g_stream));
    return FGM_CUDA_OK;
  }
  return d2h_rows_finish(C + (size_t)n0 * 16, (size_t)ldc * 4, (size_t)cols * 4, M, o_c,
                         c_pinned);
}

// Host-pointer Gemm::run (forward.rs:128-158): prep on the device, then GEMM.
static int host_linear(bool q4, const float *src, int lda, int hsz, int M, int N, int K,
                       const void *B, const void *b_scale, int group, float *C, int ldc) {
  int rc = check_gemm(M, N, K, ldc, 0, N / 16 / 4 * 4, group, q4);
  if (rc) return rc;
  if (N % 64 != 0) return fail(FGM_CUDA_EINVAL, "N=%d: linear needs N %% 64 == 0", N);
  if ((rc = check_prep(lda, M, K, hsz, 0, M, false))) return rc;
  if (M == 0) return FGM_CUDA_OK;
  if (!src || !B || !b_scale || !C) return fail(FGM_CUDA_EINVAL, "null pointer");
  std::lock_guard<std::mutex> lk(g_host_mu);
  if ((rc = ensure_device())) return rc;
  const void *dB = nullptr, *dS = nullptr;
  const size_t wbytes = q4 ? (size_t)N * K / 2 : (size_t)N * K;
  const size_t sbytes = q4 ? (size_t)(K / group) * N * 2 : (size_t)N * 4;
  if ((rc = reg_find(B, wbytes, &dB))) return rc;
  if ((rc = reg_find(b_scale, sbytes, &dS))) return rc;
  const size_t x_len = ((size_t)(M - 1) * lda + K) * 4;
  const size_t a_len = packed_len(M, K), s_len = (size_t)M * 4, c_len = (size_t)M * N * 4;
  const size_t o_a = align256(x_len), o_s = o_a + align256(a_len), o_c = o_s + align256(s_len);
  const size_t o_w = o_c + align256(c_len), o_ws = o_w + (dB ? 0 : align256(wbytes));
  const size_t o_w_end = o_ws + (dS ? 0 : align256(sbytes));
  const size_t total = o_w_end + align256((size_t)M * K);  // + row-major quantised X
  if ((rc = stage_reserve(total))) return rc;
  char *d = g_stage.d;
  const bool cacheable = dB && dS;  // registered weights: every address is stable
  const void *xsrc = nullptr;  // X is read by the prep kernel straight from host memory
  if ((rc = host_readable(src, x_len, 0, &xsrc))) return rc;
  if (!dB) {
    if ((rc = h2d(d + o_w, B, wbytes, o_w))) return rc;
    dB = d + o_w;
  } else if (!q4 && M >= tc_min_m()) {
    if ((rc = prepare_q8c(static_cast<const int8_t *>(dB), N, K, g_stream))) return rc;
  }
  if (!dS) {
    if ((rc = h2d(d + o_ws, b_scale, sbytes, o_ws))) return rc;
    dS = d + o_ws;
  }
  CUtensorMap map;
  const bool tc = !q4 && M >= tc_min_m() && find_prepared(dB, &map);
  int8_t *qa_rows = tc ? (int8_t *)(d + o_w_end) : nullptr;  // row-major quantised X
  const bool c_pinned = is_pinned(C);
  // Page-locked C: the decode GEMM stores its outputs straight into it
  // through the device mapping, so no copy-engine round trip follows the
  // kernel.  Tensor-core tiles (TMA stores) go through the device buffer.
  float *c_mapped = nullptr;
  if (c_pinned && !tc) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, C) == cudaSuccess && a.devicePointer)
      c_mapped = static_cast<float *>(a.devicePointer);
    else
      cudaGetLastError();
  }
  auto enqueue = [&]() -> int {
    int r = run_prep(static_cast<const float *>(xsrc), lda, nullptr, qa_rows, (float *)(d + o_s),
                     (int8_t *)(d + o_a), M, K, hsz, 0, M, g_stream);
    if (r) return r;
    if (tc)
      r = run_q8c_tc(M, N, K, qa_rows, K, (const float *)(d + o_s), (const float *)dS, map,
                     (float *)(d + o_c), N, 0, nullptr, 0, N / 16, g_stream);
    else
      r = run_gemm(q4, M, N, K, (const int8_t *)(d + o_a), (const float *)(d + o_s), dB, dS,
                   group, c_mapped ? c_mapped : (float *)(d + o_c), c_mapped ? ldc : N, 0,
                   nullptr, 0, N / 16, g_stream);
    if (r) return r;
    if (c_mapped) return FGM_CUDA_OK;
    return d2h_rows_enqueue(C, (size_t)ldc * 4, d + o_c, (size_t)N * 4, M, o_c, c_pinned);
  };
  if (cacheable) {
    CallKey key;
    memset(&key, 0, sizeof(key));
    key.src = src;
    key.B = B;
    key.bs = b_scale;
    key.C = C;
    key.q4 = q4;
    key.lda = lda;
    key.hsz = hsz;
    key.M = M;
    key.N = N;
    key.K = K;
    key.group = group;
    key.ldc = ldc;
    key.src_pinned = xsrc == static_cast<const void *>(src);
    key.c_pinned = c_pinned;
    rc = run_call(key, enqueue);
  } else {
    rc = enqueue();
  }
  if (rc) return rc;
  if (c_mapped) {
    FGM_TRY(cudaStreamSynchronize(g_stream));
    return FGM_CUDA_OK;
  }
  return d2h_rows_finish(C, (size_t)ldc * 4, (size_t)N * 4, M, o_c, c_pinned);
}

}  // namespace fgm

using namespace fgm;

// ===================================================================== C ABI
extern "C" {

int fgm_cuda_available(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  for (int i = 0; i < n; i++) {
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, i) == cudaSuccess && p.major == 10) return 1;
  }
  return 0;
}

int fgm_cuda_init(int device) {
  std::lock_guard<std::mutex> lk(g_dev_mu);
  int dev = pick_device(device);
  if (dev < 0) return dev;
  FGM_TRY(cudaSetDevice(dev));
  if (g_dev != dev) {
    if (g_stream) cudaStreamDestroy(g_stream);
    FGM_TRY(cudaStreamCreateWithFlags(&g_stream, cudaStreamNonBlocking));
    g_dev = dev;
  }
  return FGM_CUDA_OK;
}

const char *fgm_cuda_last_error(void) { return t_err.c_str(); }

int fgm_cuda_device_status(void) {
  DevInfo *di = nullptr;
  int rc = dev_info(&di);
  if (rc) return rc;
  FGM_TRY(cudaDeviceSynchronize());
  int v = 0;
  FGM_TRY(cudaMemcpy(&v, di->err, sizeof(int), cudaMemcpyDeviceToHost));
  if (v) {
    FGM_TRY(cudaMemset(di->err, 0, sizeof(int)));
    return fail(FGM_CUDA_ETIMEOUT, "a kernel gave up on a bounded wait (code %d)", v);
  }
  return FGM_CUDA_OK;
}

uint64_t fgm_cuda_launch_count(void) { return g_launches.load(); }

int fgm_gemm_q4g_cuda(int M, int N, int K, const int8_t *A, const float *a_scale,
                      const uint8_t *Bq, const uint16_t *b_scale, int group, float *C, int ldc,
                      int n0, int n1) {
  return host_gemm(true, M, N, K, A, a_scale, Bq, b_scale, group, C, ldc, n0, n1);
}

int fgm_gemm_q8c_cuda(int M, int N, int K, const int8_t *A, const float *a_scale,
                      const int8_t *B, const float *b_scale, float *C, int ldc, int n0, int n1) {
  return host_gemm(false, M, N, K, A, a_scale, B, b_scale, 64, C, ldc, n0, n1);
}

int fgm_linear_q4g_cuda(const float *src, int lda, int hsz, int M, int N, int K,
                        const uint8_t *Bq, const uint16_t *b_scale, int group, float *C,
                        int ldc) {
  return host_linear(true, src, lda, hsz, M, N, K, Bq, b_scale, group, C, ldc);
}

int fgm_linear_q8c_cuda(const float *src, int lda, int hsz, int M, int N, int K,
                        const int8_t *B, const float *b_scale, float *C, int ldc) {
  return host_linear(false, src, lda, hsz, M, N, K, B, b_scale, 64, C, ldc);
}

int fgm_prep_rows_cuda(const float *src, int lda, float *rot, int8_t *qa, float *qs, int8_t *pa,
                       int m, int k, int hsz, int r0, int r1) {
  int rc = check_prep(lda, m, k, hsz, r0, r1, qa != nullptr);
  if (rc) return rc;
  if (r0 >= r1) return FGM_CUDA_OK;
  if (!src || !qs || !pa) return fail(FGM_CUDA_EINVAL, "null pointer");
  std::lock_guard<std::mutex> lk(g_host_mu);
  if ((rc = ensure_device())) return rc;
  const int rend = (r1 + 15) / 16 * 16;
  // device images cover rows [0, rend) so row indices stay absolute
  const size_t x_len = ((size_t)(r1 - 1) * lda + k) * 4, rot_len = (size_t)m * k * 4;
  const size_t qa_len = (size_t)m * k, qs_len = (size_t)m * 4, pa_len = packed_len(rend, k);
  const size_t o_rot = align256(x_len), o_qa = o_rot + align256(rot_len);
  const size_t o_qs = o_qa + align256(qa_len), o_pa = o_qs + align256(qs_len);
  const size_t total = o_pa + align256(pa_len);
  if ((rc = stage_reserve(total))) return rc;
  char *d = g_stage.d;
  // only rows [r0, r1) of src are read
  if ((rc = h2d(d + (size_t)r0 * lda * 4, src + (size_t)r0 * lda,
                ((size_t)(r1 - 1 - r0) * lda + k) * 4, 0)))
    return rc;
  if (qa && r1 < m && r1 % 16 != 0) {  // tail rows of the last block come from qa
    const size_t off = (size_t)r1 * k, len = (size_t)(std::min(m, rend) - r1) * k;
    if ((rc = h2d(d + o_qa + off, qa + off, len, o_qa + off))) return rc;
  }
  rc = run_prep((const float *)d, lda, rot ? (float *)(d + o_rot) : nullptr,
                qa ? (int8_t *)(d + o_qa) : nullptr, (float *)(d + o_qs), (int8_t *)(d + o_pa),
                m, k, hsz, r0, r1, g_stream);
  if (rc) return rc;
  if (rot)
    FGM_TRY(cudaMemcpyAsync(g_stage.h + o_rot + (size_t)r0 * k * 4, d + o_rot + (size_t)r0 * k * 4,
                            (size_t)(r1 - r0) * k * 4, cudaMemcpyDeviceToHost, g_stream));
  if (qa)
    FGM_TRY(cudaMemcpyAsync(g_stage.h + o_qa + (size_t)r0 * k, d + o_qa + (size_t)r0 * k,
                            (size_t)(r1 - r0) * k, cudaMemcpyDeviceToHost, g_stream));
  FGM_TRY(cudaMemcpyAsync(g_stage.h + o_qs + (size_t)r0 * 4, d + o_qs + (size_t)r0 * 4,
                          (size_t)(r1 - r0) * 4, cudaMemcpyDeviceToHost, g_stream));
  const size_t pa0 = (size_t)(r0 / 16) * 16 * k, pan = packed_len(rend, k) - pa0;
  FGM_TRY(cudaMemcpyAsync(g_stage.h + o_pa + pa0, d + o_pa + pa0, pan, cudaMemcpyDeviceToHost,
                          g_stream));
  FGM_TRY(cudaStreamSynchronize(g_stream));
  if (rot) memcpy(rot + (size_t)r0 * k, g_stage.h + o_rot + (size_t)r0 * k * 4,
                  (size_t)(r1 - r0) * k * 4);
  if (qa) memcpy(qa + (size_t)r0 * k, g_stage.h + o_qa + (size_t)r0 * k, (size_t)(r1 - r0) * k);
  memcpy(qs + r0, g_stage.h + o_qs + (size_t)r0 * 4, (size_t)(r1 - r0) * 4);
  memcpy(pa + pa0, g_stage.h + o_pa + pa0, pan);
  return FGM_CUDA_OK;
}

int fgm_quant_act_cuda(const float *x, int rows, int k, int8_t *q, float *scale) {
  if (rows < 0 || k <= 0 || k % 64 != 0)
    return fail(FGM_CUDA_EINVAL, "quant_act needs rows >= 0 and k %% 64 == 0 (k=%d)", k);
  if (rows == 0) return FGM_CUDA_OK;
  // quantisation alone is prep with no rotation; the packed copy is discarded
  std::vector<int8_t> pa(packed_len(rows, k));
  return fgm_prep_rows_cuda(x, k, nullptr, q, scale, pa.data(), rows, k, 0, 0, rows);
}

int fgm_fwht_cuda(float *x, int n, int hsz) {
  if (hsz <= 0 || (hsz & (hsz - 1)) != 0 || n < 0 || n % hsz != 0)
    return fail(FGM_CUDA_EINVAL, "fwht needs hsz a power of two dividing n (n=%d, hsz=%d)", n,
                hsz);
  if (n == 0) return FGM_CUDA_OK;
  // rows of hsz values (padded to a multiple of 64 for the prep kernel's tiles)
  int k = hsz < 64 ? 64 : hsz;
  if (n % k != 0) k = hsz;  // cannot happen for hsz >= 64; small hsz uses k = 64 when it divides n
  if (k % 64 != 0) return fail(FGM_CUDA_EINVAL, "fwht with n=%d, hsz=%d unsupported", n, hsz);
  const int rows = n / k;
  std::vector<int8_t> qa((size_t)n), pa(packed_len(rows, k));
  std::vector<float> qs((size_t)rows);
  return fgm_prep_rows_cuda(x, k, x, qa.data(), qs.data(), pa.data(), rows, k, hsz, 0, rows);
}

int fgm_pack_a_cuda(int M, int K, const int8_t *A, int8_t *Ap) {
  if (M < 0 || K <= 0 || K % 64 != 0) return fail(FGM_CUDA_EINVAL, "pack_a: K %% 64 != 0");
  // pure data movement with no arithmetic: done on the host, like ops.c:279
  const int KB = K / 64, MB = (M + 15) / 16;
  for (int mb = 0; mb < MB; mb++)
    for (int kb = 0; kb < KB; kb++) {
      int8_t *d = Ap + ((size_t)mb * KB + kb) * 1024;
      for (int r = 0; r < 16; r++) {
        const int m = mb * 16 + r;
        if (m < M) memcpy(d + r * 64, A + (size_t)m * K + kb * 64, 64);
        else memset(d + r * 64, 0, 64);
      }
    }
  return FGM_CUDA_OK;
}

int fgm_cuda_register(const void *host, size_t bytes) {
  if (!host || !bytes) return fail(FGM_CUDA_EINVAL, "register: null pointer or zero size");
  int rc = ensure_device();
  if (rc) return rc;
  const void *d;
  return reg_upload(host, bytes, &d);
}

int fgm_cuda_unregister(const void *host) {
  std::lock_guard<std::mutex> lk(g_reg_mu);
  auto it = g_reg.find(host);
  if (it == g_reg.end()) return fail(FGM_CUDA_EINVAL, "unregister: %p not registered", host);
  release_prepared(it->second.dev);
  cudaFree(it->second.dev);
  g_reg_bytes -= it->second.bytes;
  g_reg.erase(it);
  bump_gen();
  return FGM_CUDA_OK;
}

const void *fgm_cuda_lookup(const void *host) {
  std::lock_guard<std::mutex> lk(g_reg_mu);
  auto it = g_reg.find(host);
  return it == g_reg.end() ? nullptr : it->second.dev;
}

size_t fgm_cuda_registry_bytes(void) {
  std::lock_guard<std::mutex> lk(g_reg_mu);
  return g_reg_bytes;
}

int fgm_cuda_gemm_q4g(int M, int N, int K, const int8_t *A, const float *a_scale,
                      const uint8_t *Bq, const uint16_t *b_scale, int group, float *C, int ldc,
                      int n0, int n1, void *stream) {
  int rc = check_gemm(M, N, K, ldc, n0, n1, group, true);
  if (rc) return rc;
  if (M > 0 && n0 < n1 && (!A || !a_scale || !Bq || !b_scale || !C))
    return fail(FGM_CUDA_EINVAL, "null pointer");
  return run_gemm(true, M, N, K, A, a_scale, Bq, b_scale, group, C, ldc, 0, nullptr, n0, n1,
                  (cudaStream_t)stream);
}

static int make_warm(const void *w, size_t w_bytes, const void *s, size_t s_bytes, Warm *out) {
  if ((w && !aligned16(w)) || (s && !aligned16(s)))
    return fail(FGM_CUDA_EINVAL, "warm regions must be 16-byte aligned");
  out->p[0] = w;
  out->bytes[0] = w_bytes;
  out->p[1] = s;
  out->bytes[1] = s_bytes;
  return FGM_CUDA_OK;
}

int fgm_cuda_gemm_q4g_warm(int M, int N, int K, const int8_t *A, const float *a_scale,
                           const uint8_t *Bq, const uint16_t *b_scale, int group, float *C,
                           int ldc, int n0, int n1, const void *next_w, size_t next_w_bytes,
                           const void *next_s, size_t next_s_bytes, void *stream) {
  int rc = check_gemm(M, N, K, ldc, n0, n1, group, true);
  if (rc) return rc;
  if (M > 0 && n0 < n1 && (!A || !a_scale || !Bq || !b_scale || !C))
    return fail(FGM_CUDA_EINVAL, "null pointer");
  Warm w;
  if ((rc = make_warm(next_w, next_w_bytes, next_s, next_s_bytes, &w))) return rc;
  return run_gemm(true, M, N, K, A, a_scale, Bq, b_scale, group, C, ldc, 0, nullptr, n0, n1,
                  (cudaStream_t)stream, w);
}

int fgm_cuda_gemm_q8c_warm(int M, int N, int K, const int8_t *A, const float *a_scale,
                           const int8_t *B, const float *b_scale, float *C, int ldc, int n0,
                           int n1, const void *next_w, size_t next_w_bytes, const void *next_s,
                           size_t next_s_bytes, void *stream) {
  int rc = check_gemm(M, N, K, ldc, n0, n1, 64, false);
  if (rc) return rc;
  if (M > 0 && n0 < n1 && (!A || !a_scale || !B || !b_scale || !C))
    return fail(FGM_CUDA_EINVAL, "null pointer");
  Warm w;
  if ((rc = make_warm(next_w, next_w_bytes, next_s, next_s_bytes, &w))) return rc;
  return run_gemm(false, M, N, K, A, a_scale, B, b_scale, 64, C, ldc, 0, nullptr, n0, n1,
                  (cudaStream_t)stream, w);
}

int fgm_cuda_gemm_q8c(int M, int N, int K, const int8_t *A, const float *a_scale,
                      const int8_t *B, const float *b_scale, float *C, int ldc, int n0, int n1,
                      void *stream) {
  int rc = check_gemm(M, N, K, ldc, n0, n1, 64, false);
  if (rc) return rc;
  if (M > 0 && n0 < n1 && (!A || !a_scale || !B || !b_scale || !C))
    return fail(FGM_CUDA_EINVAL, "null pointer");
  return run_gemm(false, M, N, K, A, a_scale, B, b_scale, 64, C, ldc, 0, nullptr, n0, n1,
                  (cudaStream_t)stream);
}

int fgm_cuda_prep_rows(const float *src, int lda, float *rot, int8_t *qa, float *qs, int8_t *pa,
                       int m, int k, int hsz, int r0, int r1, void *stream) {
  int rc = check_prep(lda, m, k, hsz, r0, r1, qa != nullptr);
  if (rc) return rc;
  if (r0 < r1 && (!src || !qs || !pa)) return fail(FGM_CUDA_EINVAL, "null pointer");
  return run_prep(src, lda, rot, qa, qs, pa, m, k, hsz, r0, r1, (cudaStream_t)stream);
}

static int check_linear_dev(const float *src, int lda, int hsz, int M, int N, int K, int ldc,
                            int n0, int n1, int group, bool q4, const void *B,
                            const void *b_scale, const float *C) {
  int rc = check_gemm(M, N, K, ldc, n0, n1, group, q4);
  if (rc) return rc;
  if ((rc = check_prep(lda, M, K, hsz, 0, M, false))) return rc;
  if (M > 0 && n0 < n1 && (!src || !B || !b_scale || !C))
    return fail(FGM_CUDA_EINVAL, "null pointer");
  return FGM_CUDA_OK;
}

int fgm_cuda_linear_q4g(const float *src, int lda, int hsz, int M, int N, int K,
                        const uint8_t *Bq, const uint16_t *b_scale, int group, float *C, int ldc,
                        int n0, int n1, void *stream) {
  int rc = check_linear_dev(src, lda, hsz, M, N, K, ldc, n0, n1, group, true, Bq, b_scale, C);
  if (rc) return rc;
  return run_linear(true, src, lda, hsz, M, N, K, Bq, b_scale, group, C, ldc, n0, n1,
                    (cudaStream_t)stream);
}

int fgm_cuda_linear_q8c(const float *src, int lda, int hsz, int M, int N, int K,
                        const int8_t *B, const float *b_scale, float *C, int ldc, int n0, int n1,
                        void *stream) {
  int rc = check_linear_dev(src, lda, hsz, M, N, K, ldc, n0, n1, 64, false, B, b_scale, C);
  if (rc) return rc;
  return run_linear(false, src, lda, hsz, M, N, K, B, b_scale, 64, C, ldc, n0, n1,
                    (cudaStream_t)stream);
}

int fgm_cuda_gemm_q8c_rows(int M, int N, int K, const int8_t *A, int lda, const float *a_scale,
                           const int8_t *B, const float *b_scale, float *C, int ldc, int n0,
                           int n1, void *stream) {
  int rc = check_gemm(M, N, K, ldc, n0, n1, 64, false);
  if (rc) return rc;
  if (lda < K || lda % 16) return fail(FGM_CUDA_EINVAL, "lda=%d: need lda >= K, lda %% 16 == 0", lda);
  if (M == 0 || n0 == n1) return FGM_CUDA_OK;
  if (!A || !a_scale || !B || !b_scale || !C) return fail(FGM_CUDA_EINVAL, "null pointer");
  CUtensorMap map;
  if (!find_prepared(B, &map))
    return fail(FGM_CUDA_EINVAL, "weight %p is not prepared (fgm_cuda_q8c_prepare)", (const void *)B);
  return run_q8c_tc(M, N, K, A, lda, a_scale, b_scale, map, C, ldc, 0, nullptr, n0, n1,
                    (cudaStream_t)stream);
}

int fgm_cuda_gemm_q8c_noalloc(int M, int N, int K, const int8_t *A, const float *a_scale,
                              const int8_t *B, const float *b_scale, float *C, int ldc, int n0,
                              int n1, void *stream) {
  int rc = check_gemm(M, N, K, ldc, n0, n1, 64, false);
  if (rc) return rc;
  if ((size_t)M * (size_t)K > kStaticRowsBytes)
    return fail(FGM_CUDA_EINVAL,
                "M*K=%zu bytes exceeds the static activation buffer of %zu bytes "
                "(fgm_cuda_gemm_q8c_noalloc)",
                (size_t)M * (size_t)K, kStaticRowsBytes);
  if (M == 0 || n0 == n1) return FGM_CUDA_OK;
  if (!A || !a_scale || !B || !b_scale || !C) return fail(FGM_CUDA_EINVAL, "null pointer");
  if (!aligned16(A) || !aligned16(B))
    return fail(FGM_CUDA_EINVAL, "activations and weights must be 16-byte aligned");
  CUtensorMap map;
  if (!find_prepared(B, &map))
    return fail(FGM_CUDA_EINVAL, "weight %p is not prepared (fgm_cuda_q8c_prepare)", (const void *)B);
  int8_t *rows = nullptr;
  rc = static_rows(&rows);
  if (rc) return rc;
  const cudaStream_t st = (cudaStream_t)stream;
  // The repack must stay a plain launch (no programmatic dependent launch):
  // the previous call's GEMM releases its dependents before it has read the
  // buffer, so an early-started repack could overwrite rows still in use.
  const cudaError_t e = launch_packed_to_rows(A, rows, M, K, st);
  if (e != cudaSuccess) return cuda_fail(e, "activation repack");
  count_launch();
  return run_q8c_tc(M, N, K, rows, K, a_scale, b_scale, map, C, ldc, 0, nullptr, n0, n1, st);
}

// ------------------------------------------------------- decode work list
struct WorkList {
  int dev = -1;
  int n = 0;
  WlPlan plan;
  void *mem = nullptr;
  WlParams params{};
};

static int check_work(int M, const fgm_cuda_work &w, int i, int n) {
  for (int d : w.deps)
    if (d != -1 && (d < 0 || d >= i))
      return fail(FGM_CUDA_EINVAL, "work %d: dependency %d is not an earlier entry", i, d);
  (void)n;
  auto al = [](const void *p, unsigned a) { return ((uintptr_t)p & (a - 1)) == 0; };
  if (w.kind == FGM_CUDA_WORK_PREP) {
    if (w.K <= 0 || w.K % 128 != 0 || w.K > 65536)
      return fail(FGM_CUDA_EINVAL, "work %d (prep): K=%d, need K %% 128 == 0", i, w.K);
    if (w.lda < w.K || w.lda % 4 != 0)
      return fail(FGM_CUDA_EINVAL, "work %d (prep): lda=%d, need lda >= K, lda %% 4 == 0", i,
                  w.lda);
    if (w.hsz < 0 || w.hsz > 128 || (w.hsz & (w.hsz - 1)) != 0 || (w.hsz > 0 && w.K % w.hsz))
      return fail(FGM_CUDA_EINVAL, "work %d (prep): hsz=%d, need 0 or a power of two <= 128",
                  i, w.hsz);
    if (!w.src || !w.pa || !w.qs) return fail(FGM_CUDA_EINVAL, "work %d (prep): null pointer", i);
    if (!al(w.src, 16) || !al(w.pa, 4) || !al(w.qs, 4))
      return fail(FGM_CUDA_EINVAL, "work %d (prep): src must be 16-byte, pa and qs 4-byte aligned",
                  i);
    return FGM_CUDA_OK;
  }
  if (w.kind != FGM_CUDA_WORK_Q4G && w.kind != FGM_CUDA_WORK_Q8C)
    return fail(FGM_CUDA_EINVAL, "work %d: kind %d", i, w.kind);
  const bool q4 = w.kind == FGM_CUDA_WORK_Q4G;
  if (w.K <= 0 || w.K % (q4 ? 512 : 256) != 0 || w.K > 16384)
    return fail(FGM_CUDA_EINVAL, "work %d: K=%d, need K %% %d == 0 and K <= 16384", i, w.K,
                q4 ? 512 : 256);
  if (w.N <= 0 || w.N % 16 != 0) return fail(FGM_CUDA_EINVAL, "work %d: N=%d", i, w.N);
  if (w.n0 < 0 || w.n1 <= w.n0 || w.n1 > w.N / 16)
    return fail(FGM_CUDA_EINVAL, "work %d: n-blocks [%d, %d) of %d", i, w.n0, w.n1, w.N / 16);
  if (w.ldc < w.n1 * 16) return fail(FGM_CUDA_EINVAL, "work %d: ldc=%d", i, w.ldc);
  if (q4 && (w.group != 64 && w.group != 128 && w.group != 256 && w.group != 512))
    return fail(FGM_CUDA_EINVAL, "work %d: group %d, need 64, 128, 256 or 512", i, w.group);
  if (q4 && w.K % w.group) return fail(FGM_CUDA_EINVAL, "work %d: K %% group != 0", i);
  if (!w.A || !w.a_scale || !w.B || !w.b_scale || !w.C)
    return fail(FGM_CUDA_EINVAL, "work %d: null pointer", i);
  if (!al(w.A, 16) || !al(w.B, 16) || !al(w.b_scale, q4 ? 16 : 4))
    return fail(FGM_CUDA_EINVAL, "work %d: A, B and int4 scales must be 16-byte aligned, int8 "
                "scales 4-byte aligned", i);
  (void)M;
  return FGM_CUDA_OK;
}

// ---------------------------------------------------------- row argmax
int fgm_cuda_argmax_partials(const float *C, int M, int N, int ldc, int col0, float *vals,
                             int32_t *idx, void *stream) {
  if (M < 0 || N <= 0 || ldc < N || col0 < 0)
    return fail(FGM_CUDA_EINVAL, "argmax: M=%d N=%d ldc=%d col0=%d", M, N, ldc, col0);
  if (M == 0) return FGM_CUDA_OK;
  if (!C || !vals || !idx) return fail(FGM_CUDA_EINVAL, "null pointer");
  const cudaError_t e =
      launch_argmax_partials(C, M, N, ldc, col0, vals, idx, use_pdl(), (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "argmax launch");
  count_launch();
  return FGM_CUDA_OK;
}

int fgm_cuda_argmax_parts(int N) { return N > 0 ? argmax_chunk_count(N) : 0; }

int fgm_cuda_worklist_create(int M, const fgm_cuda_work *w, int n, void **list) {
  if (!list) return fail(FGM_CUDA_EINVAL, "worklist: null handle pointer");
  *list = nullptr;
  if (M < 1 || M > 16) return fail(FGM_CUDA_EINVAL, "worklist: M=%d, need 1 <= M <= 16", M);
  if (n < 1 || n > 65536 || !w) return fail(FGM_CUDA_EINVAL, "worklist: %d entries", n);
  int rc = FGM_CUDA_OK;
  for (int i = 0; i < n; i++)
    if ((rc = check_work(M, w[i], i, n))) return rc;
  DevInfo *di = nullptr;
  if ((rc = dev_info(&di))) return rc;
  // Prep sources and GEMM outputs may live in page-locked host memory: the
  // kernel reads and writes them through their device mapping.  Everything
  // else (activations, weights, scales) must be device memory.
  auto mapped = [&](const void *ptr, bool host_ok, const char *what, int i,
                    const void **out) -> int {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, ptr) != cudaSuccess) {
      cudaGetLastError();
      return fail(FGM_CUDA_EINVAL, "work %d: %s is not CUDA-accessible memory", i, what);
    }
    if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) {
      *out = ptr;
      return FGM_CUDA_OK;
    }
    if (a.type == cudaMemoryTypeHost && host_ok && a.devicePointer) {
      *out = a.devicePointer;
      return FGM_CUDA_OK;
    }
    return fail(FGM_CUDA_EINVAL, "work %d: %s must be device memory%s", i, what,
                host_ok ? " or page-locked host memory" : "");
  };
  const int MT = M <= 8 ? 1 : 2;
  std::vector<WlItem> items((size_t)n);
  for (int i = 0; i < n; i++) {
    const fgm_cuda_work &s = w[i];
    WlItem &it = items[i];
    memset(&it, 0, sizeof(it));
    it.kind = s.kind == FGM_CUDA_WORK_Q4G ? kWlQ4 : (s.kind == FGM_CUDA_WORK_Q8C ? kWlQ8 : kWlPrep);
    it.N = s.N;
    it.K = s.K;
    it.deps[0] = s.deps[0];
    it.deps[1] = s.deps[1];
    if (it.kind == kWlPrep) {
      it.units = (M + 15) / 16 * 16;
      it.lda = s.lda;
      it.hsz = s.hsz;
      const void *src = nullptr, *pa = nullptr, *qs = nullptr;
      if ((rc = mapped(s.src, true, "src", i, &src)) || (rc = mapped(s.pa, false, "pa", i, &pa)) ||
          (rc = mapped(s.qs, false, "qs", i, &qs)))
        return rc;
      it.src = static_cast<const float *>(src);
      it.pa = static_cast<int8_t *>(const_cast<void *>(pa));
      it.qs = static_cast<float *>(const_cast<void *>(qs));
      continue;
    }
    it.gk = it.kind == kWlQ4 ? s.group / 64 : 0;
    it.nb0 = s.n0;
    it.units = s.n1 - s.n0;
    it.ldc = s.ldc;
    it.c_col0 = 0;
    const void *A = nullptr, *B = nullptr, *bs = nullptr, *as = nullptr, *Cp = nullptr;
    if ((rc = mapped(s.A, false, "A", i, &A)) || (rc = mapped(s.B, false, "B", i, &B)) ||
        (rc = mapped(s.b_scale, false, "b_scale", i, &bs)) ||
        (rc = mapped(s.a_scale, false, "a_scale", i, &as)) ||
        (rc = mapped(s.C, true, "C", i, &Cp)))
      return rc;
    it.B = static_cast<const uint8_t *>(B);
    it.b_scale = bs;
    it.a_scale = static_cast<const float *>(as);
    it.C = static_cast<float *>(const_cast<void *>(Cp));
    if (!encode_packed_a_map(&it.amap, s.A, s.K, MT * 8) ||
        (it.kind == kWlQ4 && !encode_scale_map(&it.smap, bs, s.K / s.group, s.N, 8 / it.gk)))
      return fail(FGM_CUDA_ERUNTIME, "worklist: cuTensorMapEncodeTiled failed for entry %d", i);
  }
  WorkList *wl = new WorkList();
  const char *why = worklist_plan(wl->plan, items, M, di->sms, di->smem_optin);
  if (why) {
    delete wl;
    return fail(FGM_CUDA_EINVAL, "worklist: %s", why);
  }
  // one device block: descriptors (64-byte aligned), segments, offsets, counters
  const size_t o_items = 0, b_items = sizeof(WlItem) * (size_t)n;
  const size_t o_segs = align256(o_items + b_items), b_segs = sizeof(WlSeg) * wl->plan.segs.size();
  const size_t o_off = align256(o_segs + b_segs), b_off = sizeof(int) * wl->plan.seg_off.size();
  const size_t o_cr = align256(o_off + b_off), b_cr = sizeof(WlCoopRow) * wl->plan.coop.size();
  const size_t o_co = align256(o_cr + b_cr), b_co = sizeof(int) * wl->plan.coop_n.size();
  const size_t o_cnt = align256(o_co + b_co), b_cnt = sizeof(unsigned) * ((size_t)n + 2);
  const size_t total = o_cnt + b_cnt;
  if (cudaMalloc(&wl->mem, total) != cudaSuccess) {
    cudaGetLastError();
    delete wl;
    return fail(FGM_CUDA_ENOMEM, "worklist: cudaMalloc(%zu)", total);
  }
  char *d = static_cast<char *>(wl->mem);
  for (WlSeg &sg : wl->plan.segs)  // each segment's view of its item's scales, on the device
    if (sg.kind == kWlQ4)
      sg.smap = &reinterpret_cast<const WlItem *>(d + o_items)[sg.item].smap;
  cudaError_t e = cudaMemcpy(d + o_items, items.data(), b_items, cudaMemcpyHostToDevice);
  if (e == cudaSuccess && b_segs)
    e = cudaMemcpy(d + o_segs, wl->plan.segs.data(), b_segs, cudaMemcpyHostToDevice);
  if (e == cudaSuccess)
    e = cudaMemcpy(d + o_off, wl->plan.seg_off.data(), b_off, cudaMemcpyHostToDevice);
  if (e == cudaSuccess && b_cr)
    e = cudaMemcpy(d + o_cr, wl->plan.coop.data(), b_cr, cudaMemcpyHostToDevice);
  if (e == cudaSuccess)
    e = cudaMemcpy(d + o_co, wl->plan.coop_n.data(), b_co, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemset(d + o_cnt, 0, b_cnt);
  if (e != cudaSuccess) {
    cudaFree(wl->mem);
    delete wl;
    return cuda_fail(e, "worklist upload");
  }
  cudaGetDevice(&wl->dev);
  wl->n = n;
  WlParams &p = wl->params;
  p.items = reinterpret_cast<const WlItem *>(d + o_items);
  p.n_items = n;
  p.segs = reinterpret_cast<const WlSeg *>(d + o_segs);
  p.seg_off = reinterpret_cast<const int *>(d + o_off);
  p.coop = reinterpret_cast<const WlCoopRow *>(d + o_cr);
  p.coop_n = reinterpret_cast<const int *>(d + o_co);
  p.done = reinterpret_cast<unsigned *>(d + o_cnt);
  p.ctas_done = p.done + n;
  p.abort = reinterpret_cast<int *>(p.done + n + 1);
  p.err = di->err;
  p.M = M;
  p.warps = wl->plan.warps;
  p.stages = wl->plan.stages;
  p.a_ring = wl->plan.a_ring;
  *list = wl;
  return FGM_CUDA_OK;
}

int fgm_cuda_worklist_run(void *list, void *stream) {
  if (!list) return fail(FGM_CUDA_EINVAL, "worklist: null handle");
  WorkList *wl = static_cast<WorkList *>(list);
  int dev = -1;
  FGM_TRY(cudaGetDevice(&dev));
  if (dev != wl->dev)
    return fail(FGM_CUDA_EINVAL, "worklist: created on device %d, current device is %d", wl->dev,
                dev);
  const cudaError_t e = launch_worklist(wl->params, wl->plan, use_pdl(), (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "worklist launch");
  count_launch();
  return FGM_CUDA_OK;
}

int fgm_cuda_worklist_destroy(void *list) {
  if (!list) return FGM_CUDA_OK;
  WorkList *wl = static_cast<WorkList *>(list);
  int cur = -1;
  cudaGetDevice(&cur);
  if (wl->dev >= 0) cudaSetDevice(wl->dev);
  cudaDeviceSynchronize();
  const cudaError_t e = cudaFree(wl->mem);
  if (cur >= 0) cudaSetDevice(cur);
  delete wl;
  if (e != cudaSuccess) return cuda_fail(e, "worklist free");
  return FGM_CUDA_OK;
}

int fgm_cuda_argmax_merge(const float *vals, const int32_t *idx, int M, int P, int32_t *out,
                          void *stream) {
  if (M < 0 || P <= 0) return fail(FGM_CUDA_EINVAL, "argmax merge: M=%d P=%d", M, P);
  if (M == 0) return FGM_CUDA_OK;
  if (!vals || !idx || !out) return fail(FGM_CUDA_EINVAL, "null pointer");
  const cudaError_t e = launch_argmax_merge(vals, idx, M, P, out, use_pdl(), (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "argmax merge launch");
  count_launch();
  return FGM_CUDA_OK;
}

// ------------------------------------------- decode-chain glue, attention
// The decode-step glue launches without programmatic dependent launch: each
// waits for the previous kernel to finish before its CTAs are placed.  Its
// kernels still release their own dependents at once, so a GEMM after them
// starts streaming weights early.  Measured on the config-3 step: early-
// launched glue CTAs sitting beside a running GEMM cost 8 % (2.03 vs 1.86 ms).
static bool glue_pdl() { return false; }

static int glue_done(cudaError_t e, const char *what) {
  if (e != cudaSuccess) return cuda_fail(e, what);
  count_launch();
  return FGM_CUDA_OK;
}

int fgm_cuda_rmsnorm(float *out, const float *x, const float *w, int rows, int n, float eps,
                     void *stream) {
  if (rows < 0 || n <= 0 || n > 49152)
    return fail(FGM_CUDA_EINVAL, "rmsnorm: rows=%d n=%d (need 0 < n <= 49152)", rows, n);
  if (rows == 0) return FGM_CUDA_OK;
  if (!out || !x) return fail(FGM_CUDA_EINVAL, "null pointer");
  return glue_done(launch_rmsnorm(out, x, w, rows, n, eps, glue_pdl(), (cudaStream_t)stream),
                   "rmsnorm launch");
}

int fgm_cuda_gelu_mul(float *out, const float *gate, const float *up, int rows, int n,
                      void *stream) {
  if (rows < 0 || n <= 0) return fail(FGM_CUDA_EINVAL, "gelu_mul: rows=%d n=%d", rows, n);
  if (rows == 0) return FGM_CUDA_OK;
  if (!out || !gate || !up) return fail(FGM_CUDA_EINVAL, "null pointer");
  return glue_done(launch_gelu_mul(out, gate, up, rows, n, glue_pdl(), (cudaStream_t)stream),
                   "gelu_mul launch");
}

static int elementwise(float *a, const float *b, float sc, size_t n, int op, void *stream) {
  if (n == 0) return FGM_CUDA_OK;
  if (!a || (op != 2 && !b)) return fail(FGM_CUDA_EINVAL, "null pointer");
  return glue_done(launch_elementwise(a, b, sc, n, op, glue_pdl(), (cudaStream_t)stream),
                   "elementwise launch");
}

int fgm_cuda_add(float *a, const float *b, size_t n, void *stream) {
  return elementwise(a, b, 0.0f, n, 0, stream);
}

int fgm_cuda_mul(float *a, const float *b, size_t n, void *stream) {
  return elementwise(a, b, 0.0f, n, 1, stream);
}

int fgm_cuda_scale(float *a, float s, size_t n, void *stream) {
  return elementwise(a, nullptr, s, n, 2, stream);
}

int fgm_cuda_softcap(float *x, int rows, int n, float cap, void *stream) {
  if (rows < 0 || n <= 0) return fail(FGM_CUDA_EINVAL, "softcap: rows=%d n=%d", rows, n);
  if (rows == 0) return FGM_CUDA_OK;
  if (!x) return fail(FGM_CUDA_EINVAL, "null pointer");
  return glue_done(launch_softcap(x, rows, n, cap, glue_pdl(), (cudaStream_t)stream),
                   "softcap launch");
}

int fgm_cuda_rope_table(float *cs, int positions, int head_dim, const float *inv_freq) {
  if (positions < 0 || head_dim <= 0 || head_dim % 2)
    return fail(FGM_CUDA_EINVAL, "rope_table: positions=%d head_dim=%d", positions, head_dim);
  if (positions == 0) return FGM_CUDA_OK;
  if (!cs || !inv_freq) return fail(FGM_CUDA_EINVAL, "null pointer");
  const int h = head_dim / 2;
  for (int p = 0; p < positions; p++)  // ops.c:137-139, this host's libm
    for (int j = 0; j < h; j++) {
      const float a = (float)p * inv_freq[j];
      cs[(size_t)p * head_dim + j] = cosf(a);
      cs[(size_t)p * head_dim + h + j] = sinf(a);
    }
  return FGM_CUDA_OK;
}

int fgm_cuda_rope_cs(float *x, int x_ld, int rows, int n_heads, int head_dim,
                     const float *inv_freq, const float *cs, int positions, const int *pos,
                     void *stream) {
  if (rows < 0 || n_heads <= 0 || head_dim <= 0 || head_dim % 2 || x_ld < n_heads * head_dim ||
      positions < 0)
    return fail(FGM_CUDA_EINVAL, "rope: rows=%d heads=%d head_dim=%d x_ld=%d positions=%d", rows,
                n_heads, head_dim, x_ld, positions);
  if (rows == 0) return FGM_CUDA_OK;
  if (!x || !inv_freq || !pos || (positions > 0 && !cs))
    return fail(FGM_CUDA_EINVAL, "null pointer");
  return glue_done(launch_rope(x, x_ld, rows, n_heads, head_dim, inv_freq, cs, positions, pos,
                               glue_pdl(), (cudaStream_t)stream),
                   "rope launch");
}

int fgm_cuda_rope(float *x, int x_ld, int rows, int n_heads, int head_dim, const float *inv_freq,
                  const int *pos, void *stream) {
  return fgm_cuda_rope_cs(x, x_ld, rows, n_heads, head_dim, inv_freq, nullptr, 0, pos, stream);
}

int fgm_cuda_quant_act(const float *x, int rows, int k, int8_t *q, float *scale, void *stream) {
  int rc = check_prep(k, rows, k, 0, 0, rows, true);
  if (rc) return rc;
  if (rows == 0) return FGM_CUDA_OK;
  if (!x || !q || !scale) return fail(FGM_CUDA_EINVAL, "null pointer");
  return run_prep(x, k, nullptr, q, scale, nullptr, rows, k, 0, 0, rows, (cudaStream_t)stream);
}

int fgm_cuda_store_v_t(int8_t *vt, size_t vt_stride, const int8_t *src, int src_ld, int rows,
                       int n, int slot, void *stream) {
  if (rows < 0 || n <= 0 || slot < 0 || src_ld < n)
    return fail(FGM_CUDA_EINVAL, "store_v_t: rows=%d n=%d slot=%d src_ld=%d", rows, n, slot,
                src_ld);
  if (rows == 0) return FGM_CUDA_OK;
  if (!vt || !src) return fail(FGM_CUDA_EINVAL, "null pointer");
  return glue_done(launch_store_v_t(vt, vt_stride, src, src_ld, rows, n, slot, glue_pdl(),
                                    (cudaStream_t)stream),
                   "store_v_t launch");
}

int fgm_cuda_attend_q8(float *out, int out_ld, const float *q, int q_ld, const int8_t *kc,
                       size_t kc_stride, const float *ks, size_t ks_stride, const int8_t *vt,
                       size_t vt_stride, const float *vs, size_t vs_stride, int rows, int n_heads,
                       int kv_heads, int head_dim, int start, int end, int ring, void *stream) {
  if (rows < 0 || rows > 65535 || n_heads <= 0 || kv_heads <= 0 || n_heads % kv_heads != 0)
    return fail(FGM_CUDA_EINVAL, "attend: rows=%d heads=%d kv_heads=%d", rows, n_heads, kv_heads);
  if (head_dim <= 0 || head_dim % 64 != 0 || head_dim > 512)
    return fail(FGM_CUDA_EINVAL, "attend: head_dim=%d (need a multiple of 64, at most 512)",
                head_dim);
  if (start < 0 || end <= start || ring < 0 || (ring > 0 && end - start > ring))
    return fail(FGM_CUDA_EINVAL, "attend: positions [%d, %d) ring=%d (a ring window must fit the ring)",
                start, end, ring);
  if (out_ld < n_heads * head_dim || q_ld < n_heads * head_dim)
    return fail(FGM_CUDA_EINVAL, "attend: out_ld=%d q_ld=%d < heads*head_dim", out_ld, q_ld);
  if (rows == 0) return FGM_CUDA_OK;
  if (!out || !q || !kc || !ks || !vt || !vs) return fail(FGM_CUDA_EINVAL, "null pointer");
  {  // with several rows the strides bound each cache: the window must fit
    const size_t slots = ring ? (size_t)ring : (size_t)end, kvd = (size_t)kv_heads * head_dim;
    if (rows > 1 && (slots * kvd > kc_stride || slots > ks_stride || slots > vs_stride ||
                     ((slots + 3) & ~(size_t)3) * kvd > vt_stride))
      return fail(FGM_CUDA_EINVAL, "attend: row strides shorter than the %zu slots the window "
                  "reads", slots);
  }
  DevInfo *di = nullptr;
  int rc = dev_info(&di);
  if (rc) return rc;
  AttnParams p{};
  p.out = out;
  p.out_ld = out_ld;
  p.q = q;
  p.q_ld = q_ld;
  p.kc = kc;
  p.ks = ks;
  p.vt = vt;
  p.vs = vs;
  p.kc_stride = kc_stride;
  p.ks_stride = ks_stride;
  p.vt_stride = vt_stride;
  p.vs_stride = vs_stride;
  p.n_heads = n_heads;
  p.kv_heads = kv_heads;
  p.head_dim = head_dim;
  p.start = start;
  p.end = end;
  p.ring = ring;
  p.wbase = ring ? 0 : (start & ~3);
  p.wslots = ring ? ((ring + 3) & ~3) : (((end + 3) & ~3) - p.wbase);
  if ((reinterpret_cast<uintptr_t>(kc) | reinterpret_cast<uintptr_t>(vt) | kc_stride | vt_stride) & 3)
    return fail(FGM_CUDA_EINVAL, "attend: K / V caches and their row strides must be 4-byte aligned");
  p.vec16 = ((reinterpret_cast<uintptr_t>(kc) | reinterpret_cast<uintptr_t>(vt) | kc_stride |
              vt_stride) & 15) == 0;
  if (!attend_layout(p, di->smem_optin))
    return fail(FGM_CUDA_EINVAL, "attend: %d positions, %d query heads per KV head, head_dim %d "
                "do not fit in shared memory (at most 16 heads per KV head)", end - start,
                n_heads / kv_heads, head_dim);
  return glue_done(launch_attend_q8(p, rows, glue_pdl(), di->smem_optin, (cudaStream_t)stream),
                   "attend launch");
}

int fgm_cuda_norm_prep(float *h, const float *proj, const float *w_post, const float *w_pre,
                       int rows, int n, float eps, float *qs, int8_t *pa, void *stream) {
  if (rows < 0 || n <= 0 || n % 64 != 0 || n > 12288)
    return fail(FGM_CUDA_EINVAL, "norm_prep: rows=%d n=%d (need n %% 64 == 0, n <= 12288)", rows,
                n);
  if (rows == 0) return FGM_CUDA_OK;
  if (!h || !qs || !pa) return fail(FGM_CUDA_EINVAL, "null pointer");
  if ((reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(proj) |
       reinterpret_cast<uintptr_t>(w_post) | reinterpret_cast<uintptr_t>(w_pre)) & 15)
    return fail(FGM_CUDA_EINVAL, "norm_prep: h, proj and the weights must be 16-byte aligned");
  return glue_done(launch_norm_prep(h, proj, w_post, w_pre, rows, n, eps, qs, pa, glue_pdl(),
                                    (cudaStream_t)stream),
                   "norm_prep launch");
}

int fgm_cuda_gelu_mul_prep(const float *gate, const float *up, int ld, int rows, int n,
                           float *act, float *qs, int8_t *pa, void *stream) {
  if (rows < 0 || rows > 65520 || n <= 0 || n % 64 != 0 || n > 49152 || ld < n || ld % 4 != 0)
    return fail(FGM_CUDA_EINVAL,
                "gelu_mul_prep: rows=%d n=%d ld=%d (need n %% 64 == 0, n <= 49152, ld >= n, "
                "ld %% 4 == 0)", rows, n, ld);
  if (rows == 0) return FGM_CUDA_OK;
  if (!gate || !up || !qs || !pa) return fail(FGM_CUDA_EINVAL, "null pointer");
  if ((reinterpret_cast<uintptr_t>(gate) | reinterpret_cast<uintptr_t>(up) |
       reinterpret_cast<uintptr_t>(act)) & 15)
    return fail(FGM_CUDA_EINVAL, "gelu_mul_prep: gate, up and act must be 16-byte aligned");
  return glue_done(
      launch_gelu_mul_prep(gate, up, ld, rows, n, act, qs, pa, glue_pdl(), (cudaStream_t)stream),
      "gelu_mul_prep launch");
}

int fgm_cuda_qkv_post(float *q, int q_ld, float *k, float *v, int kv_ld, int rows, int n_heads,
                      int kv_heads, int head_dim, const float *q_norm, const float *k_norm, float eps,
                      const float *inv_freq, const int *pos, int ring, int cap, int8_t *kc,
                      size_t kc_stride, float *ks, size_t ks_stride, int8_t *vt, size_t vt_stride,
                      float *vs, size_t vs_stride, void *stream) {
  return fgm_cuda_qkv_post_cs(q, q_ld, k, v, kv_ld, rows, n_heads, kv_heads, head_dim, q_norm,
                              k_norm, eps, inv_freq, nullptr, 0, pos, ring, cap, kc, kc_stride, ks,
                              ks_stride, vt, vt_stride, vs, vs_stride, stream);
}

int fgm_cuda_qkv_post_cs(float *q, int q_ld, float *k, float *v, int kv_ld, int rows,
                         int n_heads, int kv_heads, int head_dim, const float *q_norm,
                         const float *k_norm, float eps, const float *inv_freq, const float *cs,
                         int positions, const int *pos, int ring, int cap, int8_t *kc,
                         size_t kc_stride, float *ks, size_t ks_stride, int8_t *vt,
                         size_t vt_stride, float *vs, size_t vs_stride, void *stream) {
  if (positions < 0 || (positions > 0 && !cs))
    return fail(FGM_CUDA_EINVAL, "qkv_post: rope table of %d positions at %p", positions,
                (const void *)cs);
  if (cap <= 0 || (ring > 0 && ring > cap))
    return fail(FGM_CUDA_EINVAL, "qkv_post: cap=%d ring=%d (need 0 < ring <= cap)", cap, ring);
  if (rows > 1 && ((size_t)cap * kv_heads * head_dim > kc_stride || (size_t)cap > ks_stride ||
                   (size_t)cap > vs_stride ||
                   (size_t)((cap + 3) & ~3) * kv_heads * head_dim > vt_stride))
    return fail(FGM_CUDA_EINVAL, "qkv_post: row strides shorter than %d cache slots", cap);
  if (rows < 0 || n_heads <= 0 || kv_heads <= 0 || n_heads + 2 * kv_heads > 48 ||
      head_dim <= 0 || head_dim % 4 != 0 || ring < 0 || q_ld < n_heads * head_dim ||
      kv_ld < kv_heads * head_dim || q_ld % 4 != 0 || kv_ld % 4 != 0)
    return fail(FGM_CUDA_EINVAL,
                "qkv_post: rows=%d heads=%d kv_heads=%d head_dim=%d ring=%d q_ld=%d kv_ld=%d",
                rows, n_heads, kv_heads, head_dim, ring, q_ld, kv_ld);
  if (rows == 0) return FGM_CUDA_OK;
  if (!q || !k || !v || !q_norm || !k_norm || !inv_freq || !pos || !kc || !ks || !vt || !vs)
    return fail(FGM_CUDA_EINVAL, "null pointer");
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
       reinterpret_cast<uintptr_t>(v)) & 15)
    return fail(FGM_CUDA_EINVAL, "qkv_post: q, k and v must be 16-byte aligned");
  DevInfo *di = nullptr;
  int rc = dev_info(&di);
  if (rc) return rc;
  QkvParams p{q, k, v, q_ld, kv_ld, n_heads, kv_heads, head_dim, q_norm, k_norm, eps, inv_freq,
              pos, ring, cap, kc, ks, vt, vs, kc_stride, ks_stride, vt_stride, vs_stride,
              positions > 0 ? cs : nullptr, positions};
  if (qkv_post_smem(p) > di->smem_optin)
    return fail(FGM_CUDA_EINVAL, "qkv_post: %d heads of %d need too much shared memory",
                n_heads + 2 * kv_heads, head_dim);
  return glue_done(launch_qkv_post(p, rows, glue_pdl(), (cudaStream_t)stream), "qkv_post launch");
}

// ------------------------------------------------ peer memory, fused gather
int fgm_cuda_ipc_alloc(size_t bytes, void **dev_ptr) {
  if (!dev_ptr || !bytes) return fail(FGM_CUDA_EINVAL, "ipc_alloc: null pointer or zero size");
  void *d = nullptr;
  if (cudaMalloc(&d, bytes) != cudaSuccess) {
    cudaGetLastError();
    return fail(FGM_CUDA_ENOMEM, "cudaMalloc(%zu) for a shared buffer", bytes);
  }
  const cudaError_t e = cudaMemset(d, 0, bytes);
  if (e != cudaSuccess) {
    cudaFree(d);
    return cuda_fail(e, "cudaMemset");
  }
  *dev_ptr = d;
  return FGM_CUDA_OK;
}

int fgm_cuda_ipc_free(void *dev_ptr) {
  if (dev_ptr) FGM_TRY(cudaFree(dev_ptr));
  return FGM_CUDA_OK;
}

int fgm_cuda_ipc_handle(const void *dev_ptr, void *handle) {
  if (!dev_ptr || !handle) return fail(FGM_CUDA_EINVAL, "ipc_handle: null pointer");
  cudaIpcMemHandle_t h;
  FGM_TRY(cudaIpcGetMemHandle(&h, const_cast<void *>(dev_ptr)));
  static_assert(sizeof(h) == FGM_CUDA_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  return FGM_CUDA_OK;
}

int fgm_cuda_ipc_open(const void *handle, void **dev_ptr) {
  if (!dev_ptr || !handle) return fail(FGM_CUDA_EINVAL, "ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  FGM_TRY(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return FGM_CUDA_OK;
}

int fgm_cuda_ipc_close(void *dev_ptr) {
  if (dev_ptr) FGM_TRY(cudaIpcCloseMemHandle(dev_ptr));
  return FGM_CUDA_OK;
}

int fgm_cuda_gemm_q4g_gather(int M, int N, int K, const int8_t *A, const float *a_scale,
                             const uint8_t *Bq, const uint16_t *b_scale, int group, int col0,
                             int ldc, void *const *out, unsigned long long *const *sig, int rank,
                             int world, size_t slot_floats, void *stream) {
  int rc = check_gemm(M, N, K, N, 0, N / 16, group, true);
  if (rc) return rc;
  if (world < 1 || world > kMaxGatherRanks || rank < 0 || rank >= world)
    return fail(FGM_CUDA_EINVAL, "gather: rank %d of world %d (at most %d ranks)", rank, world,
                kMaxGatherRanks);
  if (M > 16) return fail(FGM_CUDA_EINVAL, "gather: M=%d > 16 (decode GEMM only)", M);
  if (col0 < 0 || col0 % 16 != 0 || ldc % 4 != 0 || col0 + N > ldc)
    return fail(FGM_CUDA_EINVAL, "gather: columns [%d, %d) of ldc=%d", col0, col0 + N, ldc);
  if (slot_floats < (size_t)M * ldc || slot_floats % 4 != 0)
    return fail(FGM_CUDA_EINVAL, "gather: slot_floats=%zu < M*ldc or not a multiple of 4",
                slot_floats);
  if (!out || !sig || !A || !a_scale || !Bq || !b_scale)
    return fail(FGM_CUDA_EINVAL, "null pointer");
  for (int q = 0; q < world; q++)
    if (!out[q] || !sig[q] || !aligned16(out[q]) || !aligned16(sig[q]))
      return fail(FGM_CUDA_EINVAL, "gather: rank %d buffers missing or unaligned", q);
  if (M == 0) return FGM_CUDA_OK;
  if (!aligned16(Bq) || !aligned16(b_scale))
    return fail(FGM_CUDA_EINVAL, "weights and int4 scales must be 16-byte aligned");
  DevInfo *di = nullptr;
  if ((rc = dev_info(&di))) return rc;
  GemvParams p{};
  p.err = di->err;
  p.M = M;
  p.N = N;
  p.K = K;
  p.group = group;
  p.A = A;
  p.a_scale = a_scale;
  p.B = Bq;
  p.b_scale = b_scale;
  p.C = static_cast<float *>(out[rank]) + col0;
  p.ldc = ldc;
  p.g.rank = rank;
  p.g.world = world;
  p.g.slot_floats = slot_floats;
  for (int q = 0; q < world; q++) {
    p.g.out[q] = static_cast<float *>(out[q]);
    p.g.sig[q] = sig[q];
  }
  const cudaError_t e =
      launch_gemv(p, N / 16, true, use_pdl(), di->sms, di->smem_optin, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "gemm_q4g_gather launch");
  count_launch();
  return FGM_CUDA_OK;
}

int fgm_cuda_q8c_prepare(const int8_t *B, int N, int K, void *stream) {
  int rc = check_gemm(1, N, K, N, 0, 0, 64, false);
  if (rc) return rc;
  if (!B || !aligned16(B)) return fail(FGM_CUDA_EINVAL, "weights must be 16-byte aligned");
  return prepare_q8c(B, N, K, (cudaStream_t)stream);
}

int fgm_cuda_q8c_release(const int8_t *B) {
  release_prepared(B);
  return FGM_CUDA_OK;
}

int fgm_cuda_gemm_q4g_acc(int M, int N, int K, const int8_t *A, const uint8_t *Bq, int group,
                          int32_t *acc, int n0, int n1, void *stream) {
  int rc = check_gemm(M, N, K, N, n0, n1, group, true);
  if (rc) return rc;
  if (M > 0 && n0 < n1 && (!A || !Bq || !acc)) return fail(FGM_CUDA_EINVAL, "null pointer");
  return run_gemm(true, M, N, K, A, nullptr, Bq, nullptr, group, nullptr, N, 0, acc, n0, n1,
                  (cudaStream_t)stream);
}

int fgm_cuda_gemm_q8c_acc(int M, int N, int K, const int8_t *A, const int8_t *B, int32_t *acc,
                          int n0, int n1, void *stream) {
  int rc = check_gemm(M, N, K, N, n0, n1, 64, false);
  if (rc) return rc;
  if (M > 0 && n0 < n1 && (!A || !B || !acc)) return fail(FGM_CUDA_EINVAL, "null pointer");
  return run_gemm(false, M, N, K, A, nullptr, B, nullptr, 64, nullptr, N, 0, acc, n0, n1,
                  (cudaStream_t)stream);
}

}  // extern "C"
