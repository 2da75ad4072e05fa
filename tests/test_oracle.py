"""Pins the CPU oracle (oracle/fgm_oracle.c) before anything is checked against it.

1. Known answers from the reference's own harness (the nibble convention).
2. The committed golden vectors, produced by the reference kernels and
   ``convert/quant.py`` (tests/golden/make_golden.py): bit-exact.
3. Live against the reference kernels compiled from source (oracle/_ref),
   where they are built and the CPU runs them.
"""
import hashlib

import numpy as np
import pytest

import harness
from fastgemma_b200 import fgm_format as F


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_nibble_convention_is_twos_complement(orc):
    # bench/kernels/vnni_test.c:62-69, literal table
    want = [0, 1, 2, 3, 4, 5, 6, 7, -8, -7, -6, -5, -4, -3, -2, -1]
    assert [orc.lib.orc_nibble(v) for v in range(16)] == want


def test_f16_widening_exact_for_every_half(orc):
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    want = h.view(np.float16).astype(np.float32)
    got = np.array([orc.lib.orc_f16_to_f32(int(v)) for v in h], np.float32)
    finite = np.isfinite(want)
    assert np.array_equal(got[finite].view(np.uint32), want[finite].view(np.uint32))
    assert np.array_equal(np.isnan(got), np.isnan(want))
    assert np.array_equal(got[np.isinf(want)], want[np.isinf(want)])


def test_cvt_saturation_matches_x86(orc):
    # _mm512_cvtps_epi32 + _mm512_cvtsepi32_epi8: RNE, INT_MIN on NaN/overflow
    cases = {2.5: 2, 3.5: 4, -2.5: -2, -3.5: -4, 0.5: 0, -0.5: 0, 127.4: 127,
             127.6: 127, 128.0: 127, -128.0: -128, -129.0: -128, 1e10: -128,
             float("inf"): -128, float("-inf"): -128, float("nan"): -128}
    for v, q in cases.items():
        assert orc.lib.orc_cvt_sat_i8(v) == q, v


def test_format_matches_reference_converter(orc, golden):
    """fgm_format's packers reproduce convert/quant.py's bytes."""
    st = np.array([0x9E3779B97F4A7C15], np.uint64)
    for (n, k) in [(16, 64), (32, 128), (48, 256)]:
        w8 = orc.xorshift(st, -127, 127, n * k).astype(np.int8).reshape(n, k)
        w4 = orc.xorshift(st, -8, 7, n * k).astype(np.int8).reshape(n, k)
        tag = f"fmt_{n}x{k}"
        assert sha(w8) == str(golden[tag + "_w8_sha"])
        assert sha(w4) == str(golden[tag + "_w4_sha"])
        assert np.array_equal(F.pack_b_tiles(w8), golden[tag + "_tiles8"])
        assert np.array_equal(F.pack_q4g(w4), golden[tag + "_tiles4"])
        assert np.array_equal(F.unpack_b_tiles(F.pack_b_tiles(w8), n, k), w8)
        assert np.array_equal(F.unpack_nibbles(F.pack_nibbles(w4.reshape(-1))), w4.reshape(-1))
        # the oracle's own unpack agrees with the converter's layout
        assert np.array_equal(orc.unpack_q4_tiles(F.pack_q4g(w4)), F.pack_b_tiles(w4))
    assert np.array_equal(st, golden["fmt_state_after"])


def test_pack_a_matches_oracle(orc):
    st = np.array([77], np.uint64)
    for m, k in [(1, 64), (15, 128), (16, 256), (17, 192), (40, 256)]:
        a = orc.xorshift(st, -128, 127, m * k).astype(np.int8).reshape(m, k)
        assert np.array_equal(F.pack_a(a), orc.pack_a(a))
        assert F.packed_a_len(m, k) == orc.pack_a(a).size


@pytest.mark.parametrize("idx", range(len(harness.VNNI_TEST_CASES)))
def test_vnni_test_cases_bit_exact(orc, golden, idx):
    case, A, a_scale, B, b_scale = list(harness.vnni_test_inputs(orc))[idx]
    kind, M, N, K, group, n0, n1 = case
    tag = f"vnni_{idx:02d}_{kind}_M{M}_N{N}_K{K}" + (f"_g{group}" if group else "")
    assert str(golden[tag + "_in_sha"]) == sha(A) + sha(B) + sha(a_scale) + sha(b_scale)
    ap = orc.pack_a(A)
    if kind == "q8c":
        c = orc.gemm_q8c(M, N, K, ap, a_scale, B, b_scale, n0=n0, n1=n1)
    else:
        c = orc.gemm_q4g(M, N, K, ap, a_scale, B, b_scale, group, n0=n0, n1=n1)
    assert sha(c) == str(golden[tag + "_C_sha"])
    if tag + "_C" in golden:
        assert np.array_equal(c.view(np.uint32), golden[tag + "_C"].view(np.uint32))


def test_gemm_test_case_bit_exact(orc, golden):
    g = harness.gemm_test_inputs(orc)
    assert str(golden["gemmtest_in_sha"]) == (sha(g["A"]) + sha(g["Bq"]) + sha(g["B8"]) +
                                              sha(g["bs4"]) + sha(g["bs8"]) + sha(g["a_scale"]))
    M, N, K, group = g["M"], g["N"], g["K"], g["group"]
    ap = orc.pack_a(g["A"])
    c4 = orc.gemm_q4g(M, N, K, ap, g["a_scale"], g["Bq"], g["bs4"], group)
    c8 = orc.gemm_q8c(M, N, K, ap, g["a_scale"], g["B8"], g["bs8"])
    c4d = orc.gemm_q4g(8, N, K, orc.pack_a(g["A"][:8]), g["a_scale"], g["Bq"], g["bs4"], group)
    assert np.array_equal(c4, golden["gemmtest_q4g_C"])
    assert np.array_equal(c8, golden["gemmtest_q8c_C"])
    assert np.array_equal(c4d[:8], golden["gemmtest_q4g_decode_C"])


def test_int32_accumulators_match_reference(orc, golden):
    st = np.array([0x51ED2701], np.uint64)
    for (kind, M, N, K) in [("q8c", 16, 128, 2048), ("q8c", 8, 64, 8192),
                            ("q4g", 16, 128, 2048), ("q4g", 5, 64, 8192)]:
        A = orc.xorshift(st, -127, 127, M * K).astype(np.int8).reshape(M, K)
        tag = f"acc_{kind}_M{M}_N{N}_K{K}"
        if kind == "q8c":
            B = orc.xorshift(st, -127, 127, N * K).astype(np.int8)
            acc = orc.gemm_q8c_acc(M, N, K, orc.pack_a(A), B)
        else:
            B = orc.xorshift(st, 0, 255, N * K // 2).astype(np.uint8)
            acc = orc.gemm_q4g_acc(M, N, K, orc.pack_a(A), B, K)[:, 0, :]
        assert str(golden[tag + "_in_sha"]) == sha(A) + sha(B)
        assert np.array_equal(acc, golden[tag + "_acc"]), tag


@pytest.mark.parametrize("idx", range(8))
def test_prep_rows_bit_exact(orc, golden, idx):
    prep_cases = [(1, 2048, 2048, 0), (8, 2048, 2048, 128), (17, 2048, 2176, 128),
                  (5, 512, 512, 8), (3, 256, 256, 16), (16, 8192, 8192, 128),
                  (2, 1024, 1024, 1024), (33, 512, 520, 64)]
    m, k, lda, hsz = prep_cases[idx]
    x = harness.prep_input(orc, m, lda, seed=1000 + idx)
    if idx == 1:
        x[3, :] = 0.0
    if idx == 0:
        x[0, :] = 0.0
        x[0, :8] = [127.0, 2.5, 3.5, -2.5, -3.5, 0.5, -0.5, 126.5]
    tag = f"prep_{idx}_m{m}_k{k}_lda{lda}_h{hsz}"
    assert sha(x) == str(golden[tag + "_in_sha"])
    rot, qa, qs, pa = orc.prep_rows(x, m, k, hsz, lda=lda)
    assert np.array_equal(qs.view(np.uint32), golden[tag + "_qs"].view(np.uint32))
    assert sha(rot) == str(golden[tag + "_rot_sha"])
    assert sha(qa) == str(golden[tag + "_qa_sha"])
    assert sha(pa) == str(golden[tag + "_pa_sha"])
    if idx == 0:
        assert list(qa[0, :8]) == [127, 2, 4, -2, -4, 0, 0, 126]  # round half to even


# ---------------------------------------------------------- live reference
@pytest.mark.parametrize("M,N,K,group,n0,n1", [
    (1, 64, 128, 64, 0, 4), (3, 128, 2048, 64, 4, 8), (8, 256, 2048, 64, 0, 16),
    (16, 128, 512, 128, 0, 8), (31, 64, 1024, 512, 0, 4), (40, 64, 256, 64, 0, 4),
    (9, 192, 8192, 64, 8, 12)])
def test_oracle_matches_reference_live_q4g(orc, ref, M, N, K, group, n0, n1):
    rng = np.random.default_rng(M * 1000 + N + K)
    A = rng.integers(-128, 128, size=(M, K), dtype=np.int8)
    bq = rng.integers(0, 256, size=N * K // 2, dtype=np.uint8)
    bs = rng.uniform(-0.02, 0.02, size=(K // group, N)).astype(np.float16)
    a_s = rng.uniform(0.001, 0.1, size=M).astype(np.float32)
    ap = orc.pack_a(A)
    c0 = np.full((M, N), 7.0, np.float32)
    c1 = c0.copy()
    orc.gemm_q4g(M, N, K, ap, a_s, bq, bs, group, c=c0, n0=n0, n1=n1)
    ref.gemm_q4g(M, N, K, ap, a_s, bq, bs, group, c=c1, n0=n0, n1=n1)
    assert np.array_equal(c0.view(np.uint32), c1.view(np.uint32))


@pytest.mark.parametrize("M,N,K,n0,n1", [
    (1, 64, 128, 0, 4), (8, 256, 2048, 4, 16), (16, 64, 8192, 0, 4),
    (33, 128, 256, 0, 8), (64, 64, 1024, 0, 4)])
def test_oracle_matches_reference_live_q8c(orc, ref, M, N, K, n0, n1):
    rng = np.random.default_rng(M * 7 + N + K)
    A = rng.integers(-128, 128, size=(M, K), dtype=np.int8)
    b = rng.integers(-128, 128, size=N * K, dtype=np.int8)
    bs = rng.uniform(0.001, 0.01, size=N).astype(np.float32)
    a_s = rng.uniform(0.001, 0.1, size=M).astype(np.float32)
    ap = orc.pack_a(A)
    c0 = np.full((M, N), -3.0, np.float32)
    c1 = c0.copy()
    orc.gemm_q8c(M, N, K, ap, a_s, b, bs, c=c0, n0=n0, n1=n1)
    ref.gemm_q8c(M, N, K, ap, a_s, b, bs, c=c1, n0=n0, n1=n1)
    assert np.array_equal(c0.view(np.uint32), c1.view(np.uint32))


@pytest.mark.parametrize("m,k,lda,hsz", [(1, 128, 128, 128), (7, 2048, 2100, 128),
                                         (16, 256, 256, 4), (20, 512, 512, 32)])
def test_oracle_matches_reference_live_prep(orc, ref, m, k, lda, hsz):
    x = np.random.default_rng(m + k).standard_normal((m, lda)).astype(np.float32)
    a = orc.prep_rows(x, m, k, hsz, lda=lda)
    b = ref.prep_rows(x, m, k, hsz, lda=lda)
    for u, v in zip(a, b):
        assert np.array_equal(u.view(np.uint8), v.view(np.uint8))


# ------------------------------------------------ decode-chain glue, attention
@pytest.mark.parametrize("n", [16, 256, 2048, 8192])
def test_glue_ops_match_reference_live(orc, ref, n):
    """rmsnorm (with and without weight), gelu_mul, add, softcap (ops.c:59-147,
    :317-352): bit-exact against the reference kernels for n a multiple of 16
    (the vector path; the reference's scalar tails call libm)."""
    rng = np.random.default_rng(n)
    x = (rng.standard_normal((3, n)) * 3).astype(np.float32)
    w = rng.standard_normal(n).astype(np.float32)
    g = (rng.standard_normal(n) * 4).astype(np.float32)
    u = rng.standard_normal(n).astype(np.float32)
    same = lambda a, b: np.array_equal(a.view(np.uint32), b.view(np.uint32))  # noqa: E731
    assert same(orc.rmsnorm(x, w, 1e-6), ref.rmsnorm(x, w, 1e-6))
    assert same(orc.rmsnorm(x, None, 1e-6), ref.rmsnorm(x, None, 1e-6))
    assert same(orc.gelu_mul(g, u), ref.gelu_mul(g, u))
    assert same(orc.add(g, u), ref.add(g, u))
    assert same(orc.softcap(g * 10, 30.0), ref.softcap(g * 10, 30.0))


@pytest.mark.parametrize("pos", [0, 7, 513, 4095])
def test_rope_matches_reference_live(orc, ref, pos):
    rng = np.random.default_rng(pos)
    nh, hd = 8, 256
    inv = (1.0 / (10000 ** (np.arange(0, hd, 2) / hd))).astype(np.float32)
    inv[-16:] = 0.0  # proportional RoPE's pass-through tail
    x = rng.standard_normal(nh * hd).astype(np.float32)
    a, b = orc.rope(x, nh, hd, inv, pos), ref.rope(x, nh, hd, inv, pos)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def _kv_cache(orc, rng, cap, kv_heads, hd):
    kc = rng.integers(-127, 128, (cap, kv_heads * hd)).astype(np.int8)
    ks = rng.uniform(0.001, 0.02, cap).astype(np.float32)
    vt = np.zeros((cap + 4) * kv_heads * hd, np.int8)
    for s in range(cap):
        orc.store_v_t(vt, rng.integers(-127, 128, kv_heads * hd).astype(np.int8), s)
    vs = rng.uniform(0.001, 0.02, cap).astype(np.float32)
    return kc, ks, vt, vs


@pytest.mark.parametrize("end,start,ring,hd", [(64, 0, 0, 256), (100, 0, 0, 256),
                                               (1024, 0, 0, 256), (1024, 17, 0, 512),
                                               (300, 40, 0, 256), (600, 500, 128, 256),
                                               (257, 129, 128, 256)])
def test_attention_matches_reference_live(orc, ref, end, start, ring, hd):
    """fgm_attend_q8_heads (ops.c:378-640): per-head int8 Q, int8 K scores,
    softmax with the Cephes exp lanes (libm expf on the tail), 16-bit split
    weights against the slot-interleaved int8 V; linear and ring caches
    (a ring window never longer than the ring, as the reference uses it)."""
    rng = np.random.default_rng(end + start + ring + hd)
    kc, ks, vt, vs = _kv_cache(orc, rng, ring or end, 2, hd)
    q = (rng.standard_normal(8 * hd) * 2).astype(np.float32)
    a = orc.attend_q8(q, kc, ks, vt, vs, 8, 2, hd, start, end, ring)
    b = ref.attend_q8(q, kc, ks, vt, vs, 8, 2, hd, start, end, ring)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_store_v_t_matches_reference_live(orc, ref):
    rng = np.random.default_rng(11)
    n, cap = 512, 37
    a, b = np.zeros((cap + 3) * n, np.int8), np.zeros((cap + 3) * n, np.int8)
    for slot in range(cap):
        src = rng.integers(-127, 128, n).astype(np.int8)
        orc.store_v_t(a, src, slot)
        ref.store_v_t(b, src, slot)
    assert np.array_equal(a, b)


def test_composed_decode_step_matches_the_reference(orc, ref):
    """The toy decode step composed from the oracle's restatements equals the
    same step composed from the reference's own kernels, bit for bit (GEMMs on
    the reference's AMX or VNNI path): the step the GPU test checks the device
    step against is the reference's step."""
    import decode_step
    if not ref.usable:
        pytest.skip("host CPU has neither AMX nor AVX-512 VNNI")
    inp = decode_step.make_inputs()
    got = decode_step.compose(orc, inp)
    want = decode_step.compose(ref, inp)
    for g, w, what in zip(got, want, ("logits", "K cache", "K scales", "V cache", "V scales")):
        assert np.array_equal(g.view(np.uint32) if g.dtype == np.float32 else g,
                              w.view(np.uint32) if w.dtype == np.float32 else w), what


@pytest.mark.parametrize("hd", [64, 256])
def test_rope_table_holds_the_references_cos_and_sin(orc, hd):
    """fgm_cuda_rope_table (host code of the CUDA library, no device work)
    against the cos / sin the oracle's rope applies (a unit vector [1 | 0]
    rotates to [cos | sin] exactly), and against the reference's own
    fgm_rope where it is built."""
    import fastgemma_b200.device as D
    from oracle.oracle import load_reference
    inv = (1.0 / (10000 ** (np.arange(0, hd, 2) / hd))).astype(np.float32)
    inv[-4:] = 0.0
    positions = 600
    tab = D.rope_table(positions, hd, inv)
    unit = np.concatenate([np.ones(hd // 2), np.zeros(hd // 2)]).astype(np.float32)
    ref = load_reference()
    for p in list(range(0, positions, 37)) + [positions - 1]:
        want = orc.rope(unit, 1, hd, inv, p)
        assert np.array_equal(tab[p].view(np.uint32), want.view(np.uint32)), p
        if ref is not None:
            assert np.array_equal(tab[p].view(np.uint32), ref.rope(unit, 1, hd, inv, p).view(np.uint32))
