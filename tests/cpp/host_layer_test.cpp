// Parity and contract checks of the C++ host layer (fastgemma_b200/host), in
// the manner of the reference's bench/kernels/gemm_test.c: seeded LCG data,
// each kernel against the scalar oracle (oracle/liboracle.so, test
// infrastructure), PASS / FAIL per case, exit status = number of failures.
//
//   host_layer_test cpu   contract checks that need no device
//   host_layer_test gpu   the kernels on the device, bit-exact against the oracle
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "fgm_host.hpp"

extern "C" {
void orc_pack_a(int M, int K, const int8_t *A, int8_t *Ap);
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
  std::printf("  %-58s %s\n", what.c_str(), ok ? "PASS" : "FAIL");
  if (!ok) failures++;
}

static uint32_t lcg = 12345;
static int rnd(int lo, int hi) {
  lcg = lcg * 1103515245u + 12345u;
  return lo + (int)((lcg >> 16) % (unsigned)(hi - lo + 1));
}

static uint16_t half_bits(float f) {  // exact for the values used here (k * 2^-10 steps)
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const int e = (int)((x >> 23) & 0xFF) - 127 + 15;
  const uint32_t mant = (x >> 13) & 0x3FFu;
  return (uint16_t)(sign | ((uint32_t)e << 10) | mant);
}

static bool same_bits(const std::vector<float> &a, const std::vector<float> &b) {
  return a.size() == b.size() && std::memcmp(a.data(), b.data(), a.size() * 4) == 0;
}

template <class F>
static bool throws_einval(F f) {
  try {
    f();
  } catch (const K::Error &e) {
    return e.status() == -1;
  }
  return false;
}

static void cpu_checks() {
  std::printf("== host layer, no device ==\n");
  // pool.rs:110-124 splits
  bool ok = true;
  for (size_t nb : {16384u, 1024u, 68u, 4u})
    for (size_t nt : {1u, 3u, 8u}) {
      size_t prev = 0;
      for (size_t t = 0; t < nt; t++) {
        auto r = C::split_gemm(nb, nt, t);
        ok &= r.first == prev && r.first % 4 == 0 && r.second % 4 == 0;
        prev = r.second;
      }
      ok &= prev == nb / 4 * 4;
    }
  report(ok, "split_gemm covers the n-blocks in groups of 4");
  // forward.rs:55-68
  setenv("FGM_WEIGHTS", "int4", 1);
  ok = C::WeightSel::from_env().kind == C::WeightSel::Lo;
  setenv("FGM_WEIGHTS", "int8", 1);
  ok &= C::WeightSel::from_env().kind == C::WeightSel::Hi;
  setenv("FGM_WEIGHTS", "auto:32", 1);
  auto s = C::WeightSel::from_env();
  ok &= s.kind == C::WeightSel::Above && s.threshold == 32;
  setenv("FGM_WEIGHTS", "auto:x", 1);
  ok &= C::WeightSel::from_env().threshold == 16;
  unsetenv("FGM_WEIGHTS");
  ok &= C::WeightSel::from_env().kind == C::WeightSel::Above;
  report(ok, "WeightSel::from_env (int4 | int8 | auto:M, default auto:16)");
  C::QLinear lo, hi;
  lo.bits = 4;
  hi.bits = 8;
  C::DualW d(lo, &hi), only(lo);
  C::WeightSel a16;
  ok = d.pick(15, a16).bits == 4 && d.pick(16, a16).bits == 8 && only.pick(64, a16).bits == 4;
  report(ok, "DualW::pick: int8 twin from 16 rows, primary otherwise");
  // contract violations throw EINVAL before any device work (lib.rs:177-178)
  std::vector<int8_t> a(16 * 64);
  std::vector<float> as(16), c(16 * 64);
  std::vector<uint8_t> bq(64 * 64 / 2);
  std::vector<uint16_t> bs(64);
  ok = throws_einval([&] { K::gemm_q4g(8, 64, 96, a, as, bq, bs, 64, c, 64, 0, 4); });
  ok &= throws_einval([&] { K::gemm_q4g(8, 64, 64, a, as, bq, bs, 64, c, 64, 0, 3); });
  ok &= throws_einval([&] { K::gemm_q4g(8, 72, 64, a, as, bq, bs, 64, c, 72, 0, 4); });
  report(ok, "gemm_q4g rejects K % 64, odd n-block ranges, N % 16");
}

static void gpu_checks() {
  std::printf("== host layer on the device (vs scalar oracle) ==\n");
  std::printf("  backend: %s\n", K::name(K::backend()));
  const int M = 40, N = 64, Kd = 256, group = 64, NB = N / 16;
  std::vector<int8_t> A((size_t)M * Kd), Ap(K::packed_a_len(M, Kd)), Ap_ref(Ap.size());
  std::vector<float> as(M);
  std::vector<uint8_t> Bq((size_t)N * Kd / 2);
  std::vector<int8_t> B8((size_t)N * Kd);
  std::vector<uint16_t> bs4((size_t)(Kd / group) * N);
  std::vector<float> bs8(N);
  for (auto &v : A) v = (int8_t)rnd(-127, 127);
  for (int i = 0; i < M; i++) as[i] = 0.002f + 0.001f * (i % 7);
  for (auto &v : Bq) v = (uint8_t)((rnd(-8, 7) & 0xF) | ((rnd(-8, 7) & 0xF) << 4));
  for (auto &v : B8) v = (int8_t)rnd(-127, 127);
  for (size_t i = 0; i < bs4.size(); i++) bs4[i] = half_bits(0.0078125f + 0.0009765625f * (i % 5));
  for (int i = 0; i < N; i++) bs8[i] = 0.003f + 0.0005f * (i % 11);

  K::pack_a(M, Kd, A, Ap);
  orc_pack_a(M, Kd, A.data(), Ap_ref.data());
  report(Ap == Ap_ref, "pack_a M=40 K=256");

  std::vector<float> Cg((size_t)M * N), Cr((size_t)M * N);
  K::gemm_q4g(M, N, Kd, Ap, as, Bq, bs4, group, Cg, N, 0, NB);
  orc_gemm_q4g(M, N, Kd, Ap.data(), as.data(), Bq.data(), bs4.data(), group, Cr.data(), N, 0, NB);
  report(same_bits(Cg, Cr), "gemm_q4g M=40 N=64 K=256 g=64 bit-exact");
  K::gemm_q8c(M, N, Kd, Ap, as, B8, bs8, Cg, N, 0, NB);
  orc_gemm_q8c(M, N, Kd, Ap.data(), as.data(), B8.data(), bs8.data(), Cr.data(), N, 0, NB);
  report(same_bits(Cg, Cr), "gemm_q8c M=40 N=64 K=256 bit-exact");
  std::vector<int8_t> Ap8(K::packed_a_len(8, Kd));
  K::pack_a(8, Kd, A, Ap8);
  std::vector<float> C8g((size_t)8 * N), C8r((size_t)8 * N);
  K::gemm_q4g(8, N, Kd, Ap8, as, Bq, bs4, group, C8g, N, 0, NB);
  orc_gemm_q4g(8, N, Kd, Ap8.data(), as.data(), Bq.data(), bs4.data(), group, C8r.data(), N, 0,
               NB);
  report(same_bits(C8g, C8r), "gemm_q4g M=8 (decode shape) bit-exact");

  // Pool::gemm over a registered weight, and Gemm::run (prep + gemm)
  C::QLinear w;
  w.bits = 4;
  w.n = N;
  w.k = Kd;
  w.q4 = Bq.data();
  w.q4_len = Bq.size();
  w.s4 = bs4.data();
  w.s4_len = bs4.size();
  w.group = group;
  w.hadamard = 128;
  C::register_linear(w);
  std::vector<float> X((size_t)M * Kd);
  for (auto &v : X) v = (float)rnd(-1000, 1000) / 250.0f;
  C::Pool pool(8);
  C::Gemm gm;
  gm.run(pool, w, X.data(), M, Kd, Cg.data());
  std::vector<float> rot((size_t)M * Kd), qs(M);
  std::vector<int8_t> qa((size_t)M * Kd), pa(K::packed_a_len(M, Kd));
  orc_prep_rows(X.data(), Kd, rot.data(), qa.data(), qs.data(), pa.data(), M, Kd, 128, 0, M);
  orc_gemm_q4g(M, N, Kd, pa.data(), qs.data(), Bq.data(), bs4.data(), group, Cr.data(), N, 0, NB);
  report(same_bits(Cg, Cr), "Gemm::run (FWHT-128, quantise, pack, q4g) bit-exact");
  C::unregister_linear(w);
  // status -> exception with the library's message
  bool threw = false;
  try {
    K::gemm_q4g(8, N, Kd, Ap8, as, Bq, bs4, 96, C8g, N, 0, NB);  // group 96: not % 64
  } catch (const K::Error &e) {
    threw = e.status() == -1 && std::string(e.what()).find("group") != std::string::npos;
  }
  report(threw, "kernel status EINVAL surfaces as fgm_kernels::Error");
}

int main(int argc, char **argv) {
  const std::string mode = argc > 1 ? argv[1] : "cpu";
  if (mode == "cpu") {
    cpu_checks();
    // without a device, backend() refuses: no CPU fallback behind the API
    unsetenv("FGM_BACKEND");
    bool threw = false;
    try {
      K::backend();
    } catch (const K::Error &e) {
      threw = e.status() == -2;
    }
    report(threw, "backend() without an sm_100 device throws ENODEV");
  } else {
    gpu_checks();
  }
  std::printf("%d failure(s)\n", failures);
  return failures;
}
