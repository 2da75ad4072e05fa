// Implementation of the C++ host layer (fgm_host.hpp) over include/fgm_cuda.h.

#include "fgm_host.hpp"

#include <cstdlib>
#include <cstring>
#include <mutex>

#include "fgm_cuda.h"

namespace fgm_kernels {

namespace {

void check(int rc, const char *what) {
  if (rc != FGM_CUDA_OK)
    throw Error(rc, std::string(what) + ": " + fgm_cuda_last_error());
}

void require(bool ok, const std::string &msg) {
  if (!ok) throw Error(FGM_CUDA_EINVAL, msg);
}

int as_int(size_t v, const char *what) {
  require(v <= 0x7fffffffu, std::string(what) + " exceeds the C ABI's int range");
  return static_cast<int>(v);
}

}  // namespace

int as_int_checked(size_t v, const char *what) { return as_int(v, what); }

const char *name(Backend b) {
  switch (b) {
    case Backend::Amx: return "amx";
    case Backend::Vnni: return "avx512-vnni";
    case Backend::Cuda: return "cuda";
  }
  return "?";
}

Backend backend() {
  static std::once_flag once;
  static Backend chosen = Backend::Cuda;
  static std::string failure;
  std::call_once(once, [] {
    const char *e = std::getenv("FGM_BACKEND");
    const std::string want = e ? e : "";
    if (want == "amx" || want == "vnni") {
      failure = "FGM_BACKEND=" + want +
                ": that backend is fgm-kernels' own C kernels; this library provides cuda only";
      return;
    }
    if (!fgm_cuda_available()) {
      failure = want == "cuda" ? "FGM_BACKEND=cuda but no CUDA sm_100 device is visible"
                               : "no CUDA sm_100 device is visible (this library provides the "
                                 "cuda backend only)";
      return;
    }
    const int rc = fgm_cuda_init(-1);
    if (rc != FGM_CUDA_OK) failure = std::string("fgm_cuda_init: ") + fgm_cuda_last_error();
  });
  if (!failure.empty()) throw Error(FGM_CUDA_ENODEV, failure);
  return chosen;
}

void pack_a(size_t m, size_t k, Slice<const int8_t> a, Slice<int8_t> ap) {
  require(k % 64 == 0, "pack_a: k % 64 != 0");
  require(a.len >= m * k, "pack_a: a shorter than m * k");
  require(ap.len >= packed_a_len(m, k), "pack_a: ap shorter than packed_a_len(m, k)");
  check(fgm_pack_a_cuda(as_int(m, "m"), as_int(k, "k"), a.ptr, ap.ptr), "pack_a");
}

static void gemm_contract(size_t m, size_t n, size_t k, size_t a_len, size_t as_len, size_t c_len,
                          size_t ldc, size_t n0, size_t n1) {
  // lib.rs:177-178 / :203-204 (debug_assert there, always checked here)
  require(k % 64 == 0 && n % 16 == 0, "gemm: need k % 64 == 0 and n % 16 == 0");
  require(n1 >= n0 && (n1 - n0) % 4 == 0, "n-block range must be a multiple of 4");
  require(a_len >= packed_a_len(m, k), "gemm: a shorter than packed_a_len(m, k)");
  require(as_len >= (m ? m : 1) || m == 0, "gemm: a_scale shorter than m");
  require(m == 0 || c_len >= (m - 1) * ldc + n, "gemm: c shorter than (m - 1) * ldc + n");
}

void gemm_q4g(size_t m, size_t n, size_t k, Slice<const int8_t> a, Slice<const float> a_scale,
              Slice<const uint8_t> bq, Slice<const f16> b_scale, size_t group, Slice<float> c,
              size_t ldc, size_t n0, size_t n1) {
  gemm_contract(m, n, k, a.len, a_scale.len, c.len, ldc, n0, n1);
  require(bq.len >= n * k / 2, "gemm_q4g: bq shorter than n * k / 2");
  require(group && b_scale.len >= k / group * n, "gemm_q4g: b_scale shorter than k/group * n");
  switch (backend()) {
    case Backend::Cuda:
      check(fgm_gemm_q4g_cuda(as_int(m, "m"), as_int(n, "n"), as_int(k, "k"), a.ptr, a_scale.ptr,
                              bq.ptr, b_scale.ptr, as_int(group, "group"), c.ptr,
                              as_int(ldc, "ldc"), as_int(n0, "n0"), as_int(n1, "n1")),
            "gemm_q4g");
      break;
    default:
      throw Error(FGM_CUDA_ENODEV, "gemm_q4g: backend not provided by this library");
  }
}

void gemm_q8c(size_t m, size_t n, size_t k, Slice<const int8_t> a, Slice<const float> a_scale,
              Slice<const int8_t> b, Slice<const float> b_scale, Slice<float> c, size_t ldc,
              size_t n0, size_t n1) {
  gemm_contract(m, n, k, a.len, a_scale.len, c.len, ldc, n0, n1);
  require(b.len >= n * k, "gemm_q8c: b shorter than n * k");
  require(b_scale.len >= n, "gemm_q8c: b_scale shorter than n");
  switch (backend()) {
    case Backend::Cuda:
      check(fgm_gemm_q8c_cuda(as_int(m, "m"), as_int(n, "n"), as_int(k, "k"), a.ptr, a_scale.ptr,
                              b.ptr, b_scale.ptr, c.ptr, as_int(ldc, "ldc"), as_int(n0, "n0"),
                              as_int(n1, "n1")),
            "gemm_q8c");
      break;
    default:
      throw Error(FGM_CUDA_ENODEV, "gemm_q8c: backend not provided by this library");
  }
}

void prep_rows(const float *src, size_t lda, float *rot, int8_t *qa, float *qs, int8_t *pa,
               size_t m, size_t k, size_t hsz, size_t r0, size_t r1) {
  backend();
  check(fgm_prep_rows_cuda(src, as_int(lda, "lda"), rot, qa, qs, pa, as_int(m, "m"),
                           as_int(k, "k"), as_int(hsz, "hsz"), as_int(r0, "r0"), as_int(r1, "r1")),
        "prep_rows");
}

void fwht(Slice<float> x, size_t hsz) {
  backend();
  check(fgm_fwht_cuda(x.ptr, as_int(x.len, "n"), as_int(hsz, "hsz")), "fwht");
}

void quant_act(Slice<const float> x, size_t rows, size_t k, Slice<int8_t> q, Slice<float> scale) {
  require(x.len >= rows * k && q.len >= rows * k && scale.len >= rows,
          "quant_act: buffers shorter than rows * k");
  backend();
  check(fgm_quant_act_cuda(x.ptr, as_int(rows, "rows"), as_int(k, "k"), q.ptr, scale.ptr),
        "quant_act");
}

void register_blob(const void *host, size_t bytes) {
  if (host && bytes) check(fgm_cuda_register(host, bytes), "register");
}

void unregister_blob(const void *host) {
  if (host) check(fgm_cuda_unregister(host), "unregister");
}

}  // namespace fgm_kernels

namespace fgm_core {

namespace k = fgm_kernels;

std::pair<size_t, size_t> split_n(size_t total, size_t nt, size_t tid) {
  const size_t per = total / nt, extra = total % nt;
  const size_t start = tid * per + (tid < extra ? tid : extra);
  return {start, start + per + (tid < extra ? 1 : 0)};
}

std::pair<size_t, size_t> split_gemm(size_t nblocks, size_t nt, size_t tid) {
  const auto ab = split_n(nblocks / 4, nt, tid);
  return {ab.first * 4, ab.second * 4};
}

// pool.rs:126-145, over the whole column range
static void run_gemm(const GemmJob &j, size_t n0, size_t n1) {
  if (n0 >= n1) return;
  const size_t m = j.m, n = j.n, kd = j.kdim;
  k::Slice<const int8_t> a(j.a, k::packed_a_len(m, kd));
  k::Slice<const float> as(j.a_scale, m ? m : 1);
  k::Slice<float> c(j.c, m * j.ldc);
  if (j.bits == 4)
    k::gemm_q4g(m, n, kd, a, as, k::Slice<const uint8_t>(j.bq, n * kd / 2),
                k::Slice<const k::f16>(j.s4, kd / j.group * n), j.group, c, j.ldc, n0, n1);
  else
    k::gemm_q8c(m, n, kd, a, as, k::Slice<const int8_t>(j.b8, n * kd),
                k::Slice<const float>(j.s8, n), c, j.ldc, n0, n1);
}

void Pool::gemm(const GemmJob &job) const { run_gemm(job, 0, job.n / 16); }

void Pool::prep(const PrepJob &job) const {
  k::prep_rows(job.src, job.lda, job.rot, job.qa, job.qs, job.pa, job.m, job.k, job.hsz, 0,
               job.m);
}

void register_linear(const QLinear &w) {
  k::register_blob(w.q4, w.q4_len);
  k::register_blob(w.q8, w.q8_len);
  k::register_blob(w.s4, w.s4_len * sizeof(k::f16));
  k::register_blob(w.s8, w.s8_len * sizeof(float));
}

void unregister_linear(const QLinear &w) {
  k::unregister_blob(w.q4);
  k::unregister_blob(w.q8);
  k::unregister_blob(w.s4);
  k::unregister_blob(w.s8);
}

WeightSel WeightSel::from_env() {
  const char *e = std::getenv("FGM_WEIGHTS");
  WeightSel s;
  if (!e) return s;
  if (std::strcmp(e, "int4") == 0) {
    s.kind = Lo;
  } else if (std::strcmp(e, "int8") == 0) {
    s.kind = Hi;
  } else if (std::strncmp(e, "auto:", 5) == 0) {
    char *end = nullptr;
    const unsigned long t = std::strtoul(e + 5, &end, 10);
    s.threshold = (end != e + 5 && *end == '\0') ? t : 16;  // unparsable -> 16, as forward.rs:62
  }
  return s;
}

const QLinear &DualW::pick(size_t m, WeightSel sel) const {
  if (has_hi_ && (sel.kind == WeightSel::Hi || (sel.kind == WeightSel::Above && m >= sel.threshold)))
    return hi_;
  return lo_;
}

void Gemm::run(const Pool &pool, const QLinear &w, const float *a, size_t m, size_t lda,
               float *out) {
  const size_t kk = w.k, n = w.n;
  // The CUDA backend runs rotate + quantise + pack and the GEMM as one call
  // (the packed rows never come back to the host); the prep/gemm pair below
  // is kept for shapes that call does not take (N not a multiple of 64).
  if (k::backend() == k::Backend::Cuda && n % 64 == 0 && m > 0) {
    const int M = k::as_int_checked(m, "m"), N = k::as_int_checked(n, "n");
    const int Kd = k::as_int_checked(kk, "k"), L = k::as_int_checked(lda, "lda");
    const int H = k::as_int_checked(w.hadamard, "hadamard");
    int rc;
    if (w.bits == 4)
      rc = fgm_linear_q4g_cuda(a, L, H, M, N, Kd, w.q4, w.s4,
                               k::as_int_checked(w.group == 0 ? 64 : w.group, "group"), out, N);
    else
      rc = fgm_linear_q8c_cuda(a, L, H, M, N, Kd, w.q8, w.s8, out, N);
    if (rc != FGM_CUDA_OK) throw k::Error(rc, std::string("Gemm::run: ") + fgm_cuda_last_error());
    return;
  }
  if (rot_.size() < m * kk) rot_.resize(m * kk);
  if (qa_.size() < m * kk) qa_.resize(m * kk);
  if (qs_.size() < (m ? m : 1)) qs_.resize(m ? m : 1);
  if (pa_.size() < k::packed_a_len(m, kk)) pa_.resize(k::packed_a_len(m, kk));
  PrepJob pj;
  pj.src = a;
  pj.lda = lda;
  pj.rot = rot_.data();
  pj.qa = qa_.data();
  pj.qs = qs_.data();
  pj.pa = pa_.data();
  pj.m = m;
  pj.k = kk;
  pj.hsz = w.hadamard;
  pool.prep(pj);
  GemmJob gj;
  gj.m = m;
  gj.n = n;
  gj.kdim = kk;
  gj.a = pa_.data();
  gj.a_scale = qs_.data();
  gj.bq = w.q4;
  gj.b8 = w.q8;
  gj.s4 = w.s4;
  gj.s8 = w.s8;
  gj.bits = w.bits;
  gj.group = w.group == 0 ? 64 : w.group;
  gj.c = out;
  gj.ldc = n;
  pool.gemm(gj);
}

}  // namespace fgm_core
