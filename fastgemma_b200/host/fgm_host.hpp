// C++ host layer of the CUDA backend: the reference's Rust crates
// fgm-kernels (src/lib.rs) and fgm-core (src/pool.rs, src/model.rs,
// src/forward.rs) restated over the C ABI of include/fgm_cuda.h, with the
// same names, argument meanings and error behaviour.  Where the Rust code
// panics (a failed assert!, a kernel status), this layer throws
// fgm_kernels::Error carrying the library's message.
//
// Only Backend::Cuda is implemented here: the AMX / VNNI arms of the
// reference are its own C kernels, which this library does not contain, so
// selecting them throws instead of falling back to anything.
#pragma once

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace fgm_kernels {

using f16 = uint16_t;  // raw IEEE half bits, as lib.rs:9

// A kernel status other than FGM_CUDA_OK, or a contract violation.
class Error : public std::runtime_error {
 public:
  Error(int status, const std::string &msg) : std::runtime_error(msg), status_(status) {}
  int status() const { return status_; }

 private:
  int status_;
};

// lib.rs:86-101 plus the CUDA arm.
enum class Backend { Amx, Vnni, Cuda };
const char *name(Backend b);

// lib.rs:112-138: decided once and cached.  FGM_BACKEND=cuda|amx|vnni forces
// the choice; unset picks cuda when an sm_100 device is visible.
Backend backend();

// lib.rs:155-157
inline size_t packed_a_len(size_t m, size_t k) { return (m + 15) / 16 * 16 * k; }

// v as the C ABI's int; throws Error(EINVAL) past INT_MAX.
int as_int_checked(size_t v, const char *what);

// A borrowed slice: pointer + element count (the Rust &[T] / &mut [T]).
template <class T>
struct Slice {
  T *ptr = nullptr;
  size_t len = 0;
  Slice() = default;
  Slice(T *p, size_t n) : ptr(p), len(n) {}
  template <class U>
  Slice(std::vector<U> &v) : ptr(v.data()), len(v.size()) {}
  template <class U>
  Slice(const std::vector<U> &v) : ptr(v.data()), len(v.size()) {}
};

// lib.rs:159-165
void pack_a(size_t m, size_t k, Slice<const int8_t> a, Slice<int8_t> ap);

// lib.rs:167-193: C[m, n] = (A int8 * a_scale) . (int4-grouped B * b_scale),
// columns [n0*16, n1*16); A tile-packed.
void gemm_q4g(size_t m, size_t n, size_t k, Slice<const int8_t> a, Slice<const float> a_scale,
              Slice<const uint8_t> bq, Slice<const f16> b_scale, size_t group, Slice<float> c,
              size_t ldc, size_t n0, size_t n1);

// lib.rs:195-217
void gemm_q8c(size_t m, size_t n, size_t k, Slice<const int8_t> a, Slice<const float> a_scale,
              Slice<const int8_t> b, Slice<const float> b_scale, Slice<float> c, size_t ldc,
              size_t n0, size_t n1);

// ops.c:293-314 through the pool (pool.rs:299-311): rotate + quantise + pack
// rows [r0, r1) of src [m, lda].
void prep_rows(const float *src, size_t lda, float *rot, int8_t *qa, float *qs, int8_t *pa,
               size_t m, size_t k, size_t hsz, size_t r0, size_t r1);

// lib.rs:51-54
void fwht(Slice<float> x, size_t hsz);
void quant_act(Slice<const float> x, size_t rows, size_t k, Slice<int8_t> q, Slice<float> scale);

// Make a weight blob resident on the device (the registry of
// fgm_cuda_register); later GEMMs naming the same host address use the
// device copy.  unregister_blob drops it.
void register_blob(const void *host, size_t bytes);
void unregister_blob(const void *host);

}  // namespace fgm_kernels

namespace fgm_core {

// pool.rs:19-34
struct GemmJob {
  size_t m = 0, n = 0, kdim = 0;
  const int8_t *a = nullptr;
  const float *a_scale = nullptr;
  const uint8_t *bq = nullptr;
  const int8_t *b8 = nullptr;
  const fgm_kernels::f16 *s4 = nullptr;
  const float *s8 = nullptr;
  uint32_t bits = 4;
  size_t group = 64;
  float *c = nullptr;
  size_t ldc = 0;
};

// pool.rs:68-79
struct PrepJob {
  const float *src = nullptr;
  size_t lda = 0;
  float *rot = nullptr;
  int8_t *qa = nullptr;
  float *qs = nullptr;
  int8_t *pa = nullptr;
  size_t m = 0, k = 0, hsz = 0;
};

// pool.rs:110-124
std::pair<size_t, size_t> split_n(size_t total, size_t nt, size_t tid);
std::pair<size_t, size_t> split_gemm(size_t nblocks, size_t nt, size_t tid);

// pool.rs: with Backend::Cuda one call covers the whole column / row range
// from the calling thread (the device parallelises it); `threads` is kept
// for the callers that size their splits by it.
class Pool {
 public:
  explicit Pool(size_t nt = 1) : nt_(nt ? nt : 1) {}
  size_t threads() const { return nt_; }
  void gemm(const GemmJob &job) const;   // pool.rs:285-295
  void prep(const PrepJob &job) const;   // pool.rs:297-311

 private:
  size_t nt_;
};

// model.rs:106-117
struct QLinear {
  uint32_t bits = 4;
  size_t n = 0, k = 0;
  const uint8_t *q4 = nullptr;
  size_t q4_len = 0;
  const int8_t *q8 = nullptr;
  size_t q8_len = 0;
  const fgm_kernels::f16 *s4 = nullptr;
  size_t s4_len = 0;
  const float *s8 = nullptr;
  size_t s8_len = 0;
  size_t group = 64;
  size_t hadamard = 0;  // Hadamard block size folded into this weight, or 0
};

// Upload a linear's blobs to the device registry (Model::load's job on this
// backend); unregister before the mapping goes away.
void register_linear(const QLinear &w);
void unregister_linear(const QLinear &w);

// forward.rs:45-68
struct WeightSel {
  enum Kind { Lo, Hi, Above } kind = Above;
  size_t threshold = 16;
  static WeightSel from_env();  // FGM_WEIGHTS=int4|int8|auto[:M], default auto:16
};

// forward.rs:26-89
class DualW {
 public:
  DualW(QLinear lo, const QLinear *hi = nullptr) : lo_(lo), has_hi_(hi != nullptr) {
    if (hi) hi_ = *hi;
  }
  const QLinear &pick(size_t m, WeightSel sel) const;
  bool has_hi() const { return has_hi_; }

 private:
  QLinear lo_, hi_;
  bool has_hi_;
};

// forward.rs:115-158: rotate, quantise, tile-pack, dispatch.  On the CUDA
// backend one fgm_linear_* call does all of it (the packed rows stay on the
// device); the host scratch below serves shapes that call does not take and
// is grown once and kept (no allocation in steady state).
class Gemm {
 public:
  void run(const Pool &pool, const QLinear &w, const float *a, size_t m, size_t lda, float *out);

 private:
  std::vector<float> rot_, qs_;
  std::vector<int8_t> qa_, pa_;
};

}  // namespace fgm_core
