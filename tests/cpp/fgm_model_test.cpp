// Checks of the C++ .fgm loader (fastgemma_b200/host/fgm_model.hpp).
//
//   fgm_model_test summary <file>   one line per tensor / linear, for the
//                                   Python reader to compare against
//   fgm_model_test errors <dir>     malformed files in <dir> must be rejected
//   fgm_model_test gpu <file>       register the file's linears and run
//                                   Gemm::run on each, bit-exact against the
//                                   scalar oracle (oracle/liboracle.so)
//
// Exit status = number of failures.
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "fgm_cuda.h"
#include "fgm_host.hpp"
#include "fgm_model.hpp"

extern "C" {
void orc_prep_rows(const float *src, int lda, float *rot, int8_t *qa, float *qs, int8_t *pa, int m,
                   int k, int hsz, int r0, int r1);
void orc_gemm_q4g(int M, int N, int K, const int8_t *Ap, const float *a_scale, const uint8_t *Bq,
                  const uint16_t *b_scale, int group, float *C, int ldc, int n0, int n1);
void orc_gemm_q8c(int M, int N, int K, const int8_t *Ap, const float *a_scale, const int8_t *B,
                  const float *b_scale, float *C, int ldc, int n0, int n1);
}

namespace K = fgm_kernels;
namespace C = fgm_core;

static int failures = 0;

static void report(bool ok, const std::string &what) {
  std::printf("  %-60s %s\n", what.c_str(), ok ? "PASS" : "FAIL");
  if (!ok) failures++;
}

static unsigned long long fnv1a(const uint8_t *p, size_t n) {
  unsigned long long h = 1469598103934665603ull;
  for (size_t i = 0; i < n; i++) {
    h ^= p[i];
    h *= 1099511628211ull;
  }
  return h;
}

static int summary(const std::string &path) {
  auto m = C::Model::open(path);
  for (const auto &kv : m->tensors()) {
    const auto &e = kv.second;
    const auto b = m->u8s(kv.first);
    std::string shape;
    for (size_t i = 0; i < e.shape.size(); i++) shape += (i ? "," : "") + std::to_string(e.shape[i]);
    std::printf("T %s %s %s %zu %zu %016llx\n", kv.first.c_str(), e.dtype.c_str(), shape.c_str(),
                e.offset, e.nbytes, fnv1a(b.ptr, b.len));
    if (e.dtype == "q4g" || e.dtype == "q8c") {
      const C::QLinear w = m->linear(kv.first);
      const size_t qlen = w.bits == 4 ? w.q4_len : w.q8_len;
      const size_t slen = w.bits == 4 ? w.s4_len : w.s8_len;
      std::printf("L %s %u %zu %zu %zu %zu %zu %zu\n", kv.first.c_str(), w.bits, w.n, w.k, w.group,
                  w.hadamard, qlen, slen);
      std::printf("D %s %d\n", kv.first.c_str(), m->dual(kv.first).has_hi() ? 1 : 0);
    }
  }
  std::printf("TOTAL %zu\n", m->total_bytes());
  const C::Json *hs = m->config().find("hidden_size");
  std::printf("CFG hidden_size %.0f\n", hs ? hs->num : -1.0);
  const C::Json *q = m->config().find("quant");
  const C::Json *ffn = q ? q->find("ffn") : nullptr;
  std::printf("CFG quant.ffn %.0f\n", ffn ? ffn->num : -1.0);
  const C::Json *gen = m->meta().find("generator");
  std::printf("META generator %s\n", gen ? gen->str.c_str() : "-");
  return 0;
}

template <class F>
static bool rejects(F f) {
  try {
    f();
  } catch (const K::Error &e) {
    return e.status() == FGM_CUDA_EINVAL;
  }
  return false;
}

static int errors(const std::string &dir) {
  for (const char *f : {"bad_magic.fgm", "short.fgm", "header_past_end.fgm", "tensor_past_end.fgm",
                        "bad_json.fgm", "missing_file.fgm"})
    report(rejects([&] { C::Model::open(dir + "/" + f); }), std::string("open rejects ") + f);
  auto m = C::Model::open(dir + "/good.fgm");
  report(rejects([&] { m->linear("no.such.tensor"); }), "linear() of a missing tensor throws");
  report(rejects([&] { m->linear("layers.0.input_layernorm.weight"); }),
         "linear() of an f32 tensor throws (non-linear dtype)");
  report(!m->has("layers.0.self_attn.q_proj.i8") && !m->dual("layers.0.self_attn.q_proj").has_hi(),
         "dual() without a twin keeps the primary");
  std::printf("%d failure(s)\n", failures);
  return failures;
}

static uint32_t lcg = 2024;
static float rnd_normalish() {
  float s = 0.0f;
  for (int i = 0; i < 4; i++) {
    lcg = lcg * 1103515245u + 12345u;
    s += (float)((lcg >> 8) & 0xFFFF) / 65536.0f;
  }
  return s - 2.0f;
}

static int gpu(const std::string &path) {
  std::printf("backend: %s\n", K::name(K::backend()));
  auto m = C::Model::open(path);
  const size_t reg = m->register_linears();
  report(reg > 0, "register_linears() made the weights resident");
  C::Pool pool;
  C::Gemm g;
  for (const auto &kv : m->tensors()) {
    if (kv.second.dtype != "q4g" && kv.second.dtype != "q8c") continue;
    const C::QLinear w = m->linear(kv.first);
    for (int M : {1, 8, 16}) {
      const int Kd = (int)w.k, N = (int)w.n;
      std::vector<float> x((size_t)M * Kd);
      for (auto &v : x) v = rnd_normalish();
      std::vector<float> got((size_t)M * N, -1.0f), want((size_t)M * N, -2.0f);
      g.run(pool, w, x.data(), M, Kd, got.data());
      std::vector<float> rot((size_t)M * Kd), qs(M);
      std::vector<int8_t> qa((size_t)M * Kd), pa(K::packed_a_len(M, Kd));
      orc_prep_rows(x.data(), Kd, rot.data(), qa.data(), qs.data(), pa.data(), M, Kd,
                    (int)w.hadamard, 0, M);
      if (w.bits == 4)
        orc_gemm_q4g(M, N, Kd, pa.data(), qs.data(), w.q4, w.s4, (int)w.group, want.data(), N, 0,
                     N / 16);
      else
        orc_gemm_q8c(M, N, Kd, pa.data(), qs.data(), w.q8, w.s8, want.data(), N, 0, N / 16);
      report(std::memcmp(got.data(), want.data(), got.size() * 4) == 0,
             kv.first + " M=" + std::to_string(M) + " bit-exact");
    }
  }
  // forward.rs:45-89: int4 below the threshold, the int8 twin from it on
  const C::DualW d = m->dual("layers.0.mlp.gate_proj");
  C::WeightSel sel;
  report(d.has_hi() && d.pick(8, sel).bits == 4 && d.pick(16, sel).bits == 8,
         "dual(): int4 at M=8, int8 twin at M=16 (auto:16)");
  m->unregister_linears();
  std::printf("%d failure(s)\n", failures);
  return failures;
}

int main(int argc, char **argv) {
  if (argc < 3) {
    std::fprintf(stderr, "usage: %s summary|errors|gpu <path>\n", argv[0]);
    return 2;
  }
  const std::string mode = argv[1], path = argv[2];
  try {
    if (mode == "summary") return summary(path);
    if (mode == "errors") return errors(path);
    if (mode == "gpu") return gpu(path);
  } catch (const std::exception &e) {
    std::printf("exception: %s\n", e.what());
    return 1;
  }
  return 2;
}
