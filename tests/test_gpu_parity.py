"""Parity of the sm_100a kernels with the reference, through the C ABI.

Bar: int32 accumulators bit-exact; f32 outputs bit-exact as well (the kernels
reproduce the reference's rounding order), which implies the north-star
tolerance of 1e-5 relative -- checked explicitly too (REL_TOL).
"""
import numpy as np
import pytest

import harness
import fastgemma_b200 as fg
import fastgemma_b200.device  # noqa: F401  (binds fg.device)
from fastgemma_b200 import fgm_format as F

pytestmark = pytest.mark.gpu
REL_TOL = 1e-5  # f32 outputs vs the reference

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", autouse=True)
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)
    from fastgemma_b200 import _lib
    assert _lib.lib().fgm_cuda_available() == 1


def D(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def assert_bits(got, want, what=""):
    got, want = np.asarray(got, np.float32), np.asarray(want, np.float32)
    assert got.shape == want.shape, (got.shape, want.shape)
    same = got.view(np.uint32) == want.view(np.uint32)
    if not same.all():
        idx = np.argwhere(~same)[:5]
        raise AssertionError(f"{what}: {int((~same).sum())} elements differ, first {idx.tolist()}: "
                             f"{got[tuple(idx[0])]} vs {want[tuple(idx[0])]}")
    denom = np.maximum(np.abs(want), 1e-30)
    assert float(np.max(np.abs(got - want) / denom, initial=0.0)) <= REL_TOL


# ---------------------------------------------------------------- golden
@pytest.mark.parametrize("idx", range(len(harness.VNNI_TEST_CASES)))
def test_reference_harness_cases_host_abi(orc, golden, idx):
    """bench/kernels/vnni_test.c's cases through the host-pointer drop-in."""
    case, A, a_scale, B, b_scale = list(harness.vnni_test_inputs(orc))[idx]
    kind, M, N, K, group, n0, n1 = case
    tag = f"vnni_{idx:02d}_{kind}_M{M}_N{N}_K{K}" + (f"_g{group}" if group else "")
    ap = F.pack_a(A)
    c = np.zeros((M, N), np.float32)
    if kind == "q8c":
        fg.gemm_q8c(M, N, K, ap, a_scale, B, b_scale, c, N, n0, n1)
    else:
        fg.gemm_q4g(M, N, K, ap, a_scale, B, b_scale, group, c, N, n0, n1)
    want = orc.gemm_q8c(M, N, K, ap, a_scale, B, b_scale, n0=n0, n1=n1) if kind == "q8c" else \
        orc.gemm_q4g(M, N, K, ap, a_scale, B, b_scale, group, n0=n0, n1=n1)
    assert_bits(c, want, tag)
    import hashlib
    assert hashlib.sha256(c.tobytes()).hexdigest() == str(golden[tag + "_C_sha"])


def test_reference_gemm_test_case(golden, orc):
    g = harness.gemm_test_inputs(orc)
    M, N, K, group = g["M"], g["N"], g["K"], g["group"]
    ap = F.pack_a(g["A"])
    c4 = np.zeros((M, N), np.float32)
    c8 = np.zeros((M, N), np.float32)
    fg.gemm_q4g(M, N, K, ap, g["a_scale"], g["Bq"], g["bs4"], group, c4, N, 0, N // 16)
    fg.gemm_q8c(M, N, K, ap, g["a_scale"], g["B8"], g["bs8"], c8, N, 0, N // 16)
    assert_bits(c4, golden["gemmtest_q4g_C"], "q4g M=40")
    assert_bits(c8, golden["gemmtest_q8c_C"], "q8c M=40")
    c4d = np.zeros((8, N), np.float32)
    fg.gemm_q4g(8, N, K, F.pack_a(g["A"][:8]), g["a_scale"], g["Bq"], g["bs4"], group, c4d, N,
                0, N // 16)
    assert_bits(c4d, golden["gemmtest_q4g_decode_C"], "q4g decode M=8")


def test_int32_accumulators_golden(orc, golden):
    st = np.array([0x51ED2701], np.uint64)
    for (kind, M, N, K) in [("q8c", 16, 128, 2048), ("q8c", 8, 64, 8192),
                            ("q4g", 16, 128, 2048), ("q4g", 5, 64, 8192)]:
        A = orc.xorshift(st, -127, 127, M * K).astype(np.int8).reshape(M, K)
        tag = f"acc_{kind}_M{M}_N{N}_K{K}"
        ap = D(F.pack_a(A))
        if kind == "q8c":
            B = orc.xorshift(st, -127, 127, N * K).astype(np.int8)
            acc = torch.zeros((M, N), dtype=torch.int32, device="cuda")
            fg.device.gemm_q8c_acc(M, N, K, ap, D(B), acc)
            got = acc.cpu().numpy()
        else:
            B = orc.xorshift(st, 0, 255, N * K // 2).astype(np.uint8)
            acc = torch.zeros((M, 1, N), dtype=torch.int32, device="cuda")
            fg.device.gemm_q4g_acc(M, N, K, ap, D(B), K, acc)
            got = acc.cpu().numpy()[:, 0, :]
        torch.cuda.synchronize()
        assert np.array_equal(got, golden[tag + "_acc"]), tag


@pytest.mark.parametrize("idx", range(8))
def test_prep_rows_golden_host_abi(orc, golden, idx):
    import hashlib
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
    rot = np.zeros((m, k), np.float32)
    qa = np.zeros((m, k), np.int8)
    qs = np.zeros(m, np.float32)
    pa = np.zeros(F.packed_a_len(m, k), np.int8)
    fg.prep_rows(x, lda, rot, qa, qs, pa, m, k, hsz, 0, m)
    sha = lambda a: hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()  # noqa: E731
    assert np.array_equal(qs.view(np.uint32), golden[tag + "_qs"].view(np.uint32))
    assert sha(rot) == str(golden[tag + "_rot_sha"])
    assert sha(qa) == str(golden[tag + "_qa_sha"])
    assert sha(pa) == str(golden[tag + "_pa_sha"])


# ------------------------------------------------- BASELINE decode shapes
DECODE = [(2048, 2048), (2048, 512), (2048, 16384), (8192, 2048)]  # (K, N): q/o, kv, gate_up, down


@pytest.mark.parametrize("M", [1, 2, 4, 8, 16])
@pytest.mark.parametrize("K,N", DECODE)
def test_decode_q4g_shapes_bit_exact(orc, M, K, N):
    """BASELINE config 1 shapes: f32 outputs and int32 group accumulators."""
    rng = np.random.default_rng(M * 100003 + K + N)
    x = rng.standard_normal((M, K), dtype=np.float32)
    bq, s = F.synth_q4g(N, K, 64, M + K + N, structured=False)
    _, _, qs, pa = orc.prep_rows(x, M, K, 0)
    xd, pad, qsd = D(x), torch.empty(pa.size, dtype=torch.int8, device="cuda"), \
        torch.empty(M, dtype=torch.float32, device="cuda")
    fg.device.prep_rows(xd, K, qsd, pad, M, K, 0)
    c = torch.full((M, N), float("nan"), device="cuda")
    bqd, sd = D(bq), D(s.view(np.uint16))
    fg.device.gemm_q4g(M, N, K, pad, qsd, bqd, sd, 64, c)
    acc = torch.zeros((M, K // 64, N), dtype=torch.int32, device="cuda")
    fg.device.gemm_q4g_acc(M, N, K, pad, bqd, 64, acc)
    torch.cuda.synchronize()
    assert np.array_equal(pad.cpu().numpy(), pa)
    assert np.array_equal(qsd.cpu().numpy().view(np.uint32), qs.view(np.uint32))
    assert_bits(c.cpu().numpy(), orc.gemm_q4g(M, N, K, pa, qs, bq, s, 64), f"q4g M={M} {K}x{N}")
    if N <= 2048:
        assert np.array_equal(acc.cpu().numpy(), orc.gemm_q4g_acc(M, N, K, pa, bq, 64))


def test_warm_entries_change_no_result(orc):
    """The L2-warming GEMM entries give the plain entries' bits, for a chain
    where each launch prefetches the next one's weights (the last one none),
    and reject unaligned regions."""
    rng = np.random.default_rng(5)
    M, K = 8, 2048
    x = rng.standard_normal((M, K), dtype=np.float32)
    _, _, qs, pa = orc.prep_rows(x, M, K, 0)
    pad, qsd = D(pa), D(qs)
    chain = [F.synth_q4g(N, K, 64, 90 + N, structured=False) for N in (2048, 512, 16384)]
    dev = [(D(bq), D(s.view(np.uint16))) for bq, s in chain]
    for j, ((bq, s), (bqd, sd)) in enumerate(zip(chain, dev)):
        N = s.shape[1]
        c = torch.full((M, N), float("nan"), device="cuda")
        nxt = dev[j + 1] if j + 1 < len(dev) else None
        fg.device.gemm_q4g_warm(M, N, K, pad, qsd, bqd, sd, 64, c, nxt)
        torch.cuda.synchronize()
        assert_bits(c.cpu().numpy(), orc.gemm_q4g(M, N, K, pa, qs, bq, s, 64), f"warm q4g {N}")
    b, s8 = F.synth_q8c(1024, K, 3)
    a_s = rng.uniform(0.001, 0.05, size=M).astype(np.float32)
    c = torch.full((M, 1024), float("nan"), device="cuda")
    fg.device.gemm_q8c_warm(M, 1024, K, pad, D(a_s), D(b), D(s8), c, dev[0])
    torch.cuda.synchronize()
    assert_bits(c.cpu().numpy(), orc.gemm_q8c(M, 1024, K, pa, a_s, b, s8), "warm q8c")
    from fastgemma_b200 import _lib
    bqd, sd = dev[0]
    with pytest.raises(_lib.FgmCudaError, match="16-byte"):
        fg.device.gemm_q4g_warm(M, 2048, K, pad, qsd, bqd, sd, 64, c, (bqd[1:], None))


@pytest.mark.parametrize("M,K,N", [(1, 2048, 512), (8, 2048, 2048), (16, 8192, 256),
                                   (17, 2048, 256), (64, 1024, 512), (256, 2048, 512),
                                   (256, 8192, 256)])
def test_q8c_shapes_bit_exact(orc, M, K, N):
    rng = np.random.default_rng(M + K * 3 + N)
    A = rng.integers(-127, 128, size=(M, K), dtype=np.int8)
    b, s = F.synth_q8c(N, K, M + N)
    a_s = rng.uniform(0.001, 0.05, size=M).astype(np.float32)
    pa = F.pack_a(A)
    c = torch.full((M, N), float("nan"), device="cuda")
    pad, bd = D(pa), D(b)
    fg.device.gemm_q8c(M, N, K, pad, D(a_s), bd, D(s), c)
    acc = torch.zeros((M, N), dtype=torch.int32, device="cuda")
    fg.device.gemm_q8c_acc(M, N, K, pad, bd, acc)
    torch.cuda.synchronize()
    assert_bits(c.cpu().numpy(), orc.gemm_q8c(M, N, K, pa, a_s, b, s), f"q8c M={M}")
    assert np.array_equal(acc.cpu().numpy(), orc.gemm_q8c_acc(M, N, K, pa, b))


@pytest.mark.parametrize("group", [128, 256, 512, 2048])
@pytest.mark.parametrize("M", [3, 16, 33])
def test_q4g_group_sizes_and_row_blocks(orc, group, M):
    K, N = 2048, 256
    rng = np.random.default_rng(group + M)
    A = rng.integers(-128, 128, size=(M, K), dtype=np.int8)
    bq, s = F.synth_q4g(N, K, group, group * 7 + M)
    a_s = rng.uniform(0.001, 0.05, size=M).astype(np.float32)
    pa = F.pack_a(A)
    c = torch.zeros((M, N), device="cuda")
    fg.device.gemm_q4g(M, N, K, D(pa), D(a_s), D(bq), D(s.view(np.uint16)), group, c)
    torch.cuda.synchronize()
    assert_bits(c.cpu().numpy(), orc.gemm_q4g(M, N, K, pa, a_s, bq, s, group))


@pytest.mark.parametrize("group", [64, 512, 4096, 8192])
def test_q4g_extreme_group_sums(orc, group):
    """Scale-group sums at and past 2^22 (every product +1024 or -1016): the
    kernel's exact int32 -> f32 conversion covers groups of up to 4096
    values, larger groups take the converter; both must match exactly."""
    M, K, N = 3, 8192, 64
    A = np.full((M, K), -128, np.int8)
    A[1] = 127
    A[2, 1::2] = 127
    bq = np.full(N * K // 2, 0x88, np.uint8)  # every weight -8
    s = np.full((K // group, N), 1.0, np.float16)
    a_s = np.ones(M, np.float32)
    pa = F.pack_a(A)
    c = torch.zeros((M, N), device="cuda")
    fg.device.gemm_q4g(M, N, K, D(pa), D(a_s), D(bq), D(s.view(np.uint16)), group, c)
    torch.cuda.synchronize()
    assert_bits(c.cpu().numpy(), orc.gemm_q4g(M, N, K, pa, a_s, bq, s, group))


def test_partial_range_ldc_and_untouched(orc):
    """Only rows < M and columns [n0*16, n1*16) are written (amx_gemm.c:333)."""
    M, N, K, n0, n1, ldc = 5, 512, 1024, 8, 20, 600
    rng = np.random.default_rng(5)
    pa = F.pack_a(rng.integers(-128, 128, size=(M, K), dtype=np.int8))
    bq, s = F.synth_q4g(N, K, 64, 5)
    b8, s8 = F.synth_q8c(N, K, 6)
    a_s = rng.uniform(0.001, 0.05, size=M).astype(np.float32)
    for q4 in (True, False):
        c = torch.full((M + 2, ldc), -7.0, device="cuda")
        if q4:
            fg.device.gemm_q4g(M, N, K, D(pa), D(a_s), D(bq), D(s.view(np.uint16)), 64, c, ldc,
                               n0, n1)
        else:
            fg.device.gemm_q8c(M, N, K, D(pa), D(a_s), D(b8), D(s8), c, ldc, n0, n1)
        torch.cuda.synchronize()
        got = c.cpu().numpy()
        want = np.full((M + 2, ldc), -7.0, np.float32)
        if q4:
            orc.gemm_q4g(M, N, K, pa, a_s, bq, s, 64, c=want, ldc=ldc, n0=n0, n1=n1)
        else:
            orc.gemm_q8c(M, N, K, pa, a_s, b8, s8, c=want, ldc=ldc, n0=n0, n1=n1)
        assert_bits(got, want, "partial range")


@pytest.mark.parametrize("pinned", [True, False])
def test_host_entries_partial_range_into_host_c(orc, pinned):
    """The reference-facing host entries (fgm_gemm_q4g_cuda / _q8c_cuda,
    fgm_linear_q4g_cuda) write only rows < M and columns [n0*16, n1*16) of a
    host C with ldc > N -- page-locked C is stored to directly by the decode
    GEMM, pageable C through the copy-back -- on repeated calls (the third
    replays the call's cached graph)."""
    from fastgemma_b200 import _lib
    M, N, K, n0, n1, ldc = 5, 512, 1024, 8, 20, 600
    rng = np.random.default_rng(8)
    pa = F.pack_a(rng.integers(-128, 128, size=(M, K), dtype=np.int8))
    bq, s = F.synth_q4g(N, K, 64, 5)
    b8, s8 = F.synth_q8c(N, K, 6)
    a_s = rng.uniform(0.001, 0.05, size=M).astype(np.float32)

    def host_c():
        t = torch.full((M + 2, ldc), -7.0)
        return t.pin_memory() if pinned else t

    for q4 in (True, False):
        want = np.full((M + 2, ldc), -7.0, np.float32)
        if q4:
            orc.gemm_q4g(M, N, K, pa, a_s, bq, s, 64, c=want, ldc=ldc, n0=n0, n1=n1)
        else:
            orc.gemm_q8c(M, N, K, pa, a_s, b8, s8, c=want, ldc=ldc, n0=n0, n1=n1)
        for _ in range(3):  # plain, captured, replayed
            c = host_c()
            if q4:
                _lib.call("fgm_gemm_q4g_cuda", M, N, K, pa.ctypes.data, a_s.ctypes.data,
                          bq.ctypes.data, s.ctypes.data, 64, c.data_ptr(), ldc, n0, n1)
            else:
                _lib.call("fgm_gemm_q8c_cuda", M, N, K, pa.ctypes.data, a_s.ctypes.data,
                          b8.ctypes.data, s8.ctypes.data, c.data_ptr(), ldc, n0, n1)
            assert_bits(c.numpy(), want, f"host entry q4={q4} pinned={pinned}")
    x = F.synth_x(M, K, 9)
    _, _, qs, pa2 = orc.prep_rows(x, M, K, 0)
    want = np.full((M + 2, ldc), -7.0, np.float32)
    orc.gemm_q4g(M, N, K, pa2, qs, bq, s, 64, c=want, ldc=ldc)
    for _ in range(2):
        c = host_c()
        _lib.call("fgm_linear_q4g_cuda", x.ctypes.data, K, 0, M, N, K, bq.ctypes.data,
                  s.ctypes.data, 64, c.data_ptr(), ldc)
        assert_bits(c.numpy(), want, f"linear pinned={pinned}")


def test_config0_full_size_bit_exact(orc):
    """BASELINE config 0 shape at full size: M=8, N=8192, K=2048, int4 g64."""
    M, N, K = 8, 8192, 2048
    x = F.synth_x(M, K, 11)
    bq, s = F.synth_q4g(N, K, 64, 12, structured=False)
    c = np.zeros((M, N), np.float32)
    fg.linear_q4g(x, K, 0, M, N, K, bq, s, 64, c, N)
    _, _, qs, pa = orc.prep_rows(x, M, K, 0)
    assert_bits(c, orc.gemm_q4g(M, N, K, pa, qs, bq, s, 64), "config 0")


def test_lm_head_full_width_sampled(orc):
    """N = 262144 LM head at M = 8: every n-block computed on the device, a
    spread of column ranges checked against the oracle, and the full output
    equal to the concatenation of independently computed column shards."""
    M, N, K = 8, 262144, 2048
    x = F.synth_x(M, K, 21)
    bq, s = F.synth_q4g(N, K, 64, 22, structured=False)
    _, _, qs, pa = orc.prep_rows(x, M, K, 0)
    pad, qsd, bqd, sd = D(pa), D(qs), D(bq), D(s.view(np.uint16))
    full = torch.empty((M, N), device="cuda")
    fg.device.gemm_q4g(M, N, K, pad, qsd, bqd, sd, 64, full)
    shards = torch.empty((M, N), device="cuda")
    nb = N // 16
    for r in range(8):  # column shards as an 8-way split would cut them
        a, b = r * nb // 8 // 4 * 4, (r + 1) * nb // 8 // 4 * 4
        fg.device.gemm_q4g(M, N, K, pad, qsd, bqd, sd, 64, shards, N, a, b)
    torch.cuda.synchronize()
    full_h = full.cpu().numpy()
    assert np.array_equal(full_h.view(np.uint32), shards.cpu().numpy().view(np.uint32))
    for a in (0, 4, 4096, 8188, 16380):
        want = np.zeros((M, N), np.float32)
        orc.gemm_q4g(M, N, K, pa, qs, bq, s, 64, c=want, n0=a, n1=a + 4)
        assert_bits(full_h[:, a * 16:(a + 4) * 16], want[:, a * 16:(a + 4) * 16], f"nb {a}")


def test_linear_host_path_matches_oracle(orc):
    """Gemm::run drop-in (host X -> prep -> GEMM -> host C) with a Hadamard."""
    for (M, K, N, hsz, q4) in [(3, 2048, 512, 128, True), (16, 8192, 256, 128, True),
                               (8, 2048, 256, 0, False), (40, 1024, 128, 64, False)]:
        x = F.synth_x(M, K, M + K)
        _, _, qs, pa = orc.prep_rows(x, M, K, hsz)
        c = np.zeros((M, N), np.float32)
        if q4:
            bq, s = F.synth_q4g(N, K, 64, N)
            fg.linear_q4g(x, K, hsz, M, N, K, bq, s, 64, c, N)
            want = orc.gemm_q4g(M, N, K, pa, qs, bq, s, 64)
        else:
            b, s = F.synth_q8c(N, K, N)
            fg.linear_q8c(x, K, hsz, M, N, K, b, s, c, N)
            want = orc.gemm_q8c(M, N, K, pa, qs, b, s)
        assert_bits(c, want, f"linear M={M} K={K} hsz={hsz}")


def test_linear_host_repeated_calls_replay_and_invalidate(orc):
    """Repeating a host-pointer call with the same buffers replays a cached
    graph (third call on): results must follow the new contents of X every
    time, and re-registering changed weights at the same address must drop
    the cached graphs."""
    M, K, N, hsz = 8, 2048, 512, 128
    bq, s = F.synth_q4g(N, K, 64, 77)
    s = np.ascontiguousarray(s)
    fg.register(bq)
    fg.register(s)
    try:
        pinned_x = torch.empty((M, K), dtype=torch.float32).pin_memory()
        pinned_c = torch.empty((M, N), dtype=torch.float32).pin_memory()
        x_np = np.zeros((M, K), np.float32)
        c_np = np.zeros((M, N), np.float32)
        rng = np.random.default_rng(8)
        for i in range(5):
            for x_buf, c_buf, arr in ((x_np, c_np, None), (pinned_x.numpy(), pinned_c.numpy(), 1)):
                x_buf[:] = rng.standard_normal((M, K)).astype(np.float32)
                fg.linear_q4g(x_buf, K, hsz, M, N, K, bq, s, 64, c_buf, N)
                _, _, qs, pa = orc.prep_rows(x_buf, M, K, hsz)
                assert_bits(c_buf, orc.gemm_q4g(M, N, K, pa, qs, bq, s, 64), f"call {i} {arr}")
            if i == 2:  # new weights at the same host address
                fg.unregister(bq)
                bq[:] = F.synth_q4g(N, K, 64, 78)[0]
                fg.register(bq)
    finally:
        fg.unregister(bq)
        fg.unregister(s)


# (M, K, N, hsz, group, lda - K): decode and prefill row counts, Hadamard
# sizes from none to 2048, padded and unaligned row pitches
LINEAR_CASES = [(1, 2048, 512, 0, 64, 0), (8, 2048, 2048, 128, 64, 4), (3, 192, 128, 64, 64, 0),
                (16, 1024, 256, 128, 128, 8), (13, 3072, 256, 16, 64, 0),
                (8, 8192, 256, 128, 64, 0), (5, 2048, 256, 1024, 256, 0),
                (8, 2048, 256, 8, 64, 0), (2, 4096, 128, 2, 512, 0), (9, 64, 64, 32, 64, 0),
                (8, 2048, 256, 128, 64, 1), (20, 2048, 256, 128, 64, 0),
                (4, 16384, 128, 128, 64, 0), (6, 4096, 128, 2048, 64, 0)]


@pytest.mark.parametrize("M,K,N,hsz,group,pad", LINEAR_CASES)
def test_linear_device_matches_prep_then_gemm(orc, M, K, N, hsz, group, pad):
    """fgm_cuda_linear_q4g / _q8c (Gemm::run on device buffers) against the
    oracle's prep_rows followed by its GEMM: bit-exact f32 in the written
    column range, untouched elsewhere."""
    lda = K + pad
    rng = np.random.default_rng(M * 7 + K + hsz + pad)
    x = (rng.standard_normal((M, lda)) * rng.uniform(0.1, 4, size=(M, 1))).astype(np.float32)
    if M > 2:
        x[1] = 0  # an all-zero row quantises with scale 1
    _, _, qs, pa = orc.prep_rows(x, M, K, hsz, lda=lda)
    bq, s4 = F.synth_q4g(N, K, group, N + K)
    b8, s8 = F.synth_q8c(N, K, N + 3)
    ldc, n0, n1 = N + 16, (4 if N >= 128 else 0), N // 16
    xd = D(x)
    c4 = torch.full((M, ldc), -5.0, device="cuda")
    c8 = torch.full((M, ldc), -5.0, device="cuda")
    fg.device.linear_q4g(xd, lda, hsz, M, N, K, D(bq), D(s4), group, c4, ldc, n0, n1)
    fg.device.linear_q8c(xd, lda, hsz, M, N, K, D(b8), D(s8), c8, ldc, n0, n1)
    torch.cuda.synchronize()
    from fastgemma_b200 import _lib
    assert _lib.lib().fgm_cuda_device_status() == 0
    want4 = np.full((M, ldc), -5.0, np.float32)
    orc.gemm_q4g(M, N, K, pa, qs, bq, s4, group, c=want4, ldc=ldc, n0=n0, n1=n1)
    assert_bits(c4.cpu().numpy(), want4, f"linear_q4g M={M} K={K} hsz={hsz}")
    want8 = np.full((M, ldc), -5.0, np.float32)
    orc.gemm_q8c(M, N, K, pa, qs, b8, s8, c=want8, ldc=ldc, n0=n0, n1=n1)
    assert_bits(c8.cpu().numpy(), want8, f"linear_q8c M={M} K={K} hsz={hsz}")


def test_linear_device_special_values(orc):
    """Rows the x86 conversion pair treats specially (ops.c:186-197): a
    denormal maximum (1/s overflows to inf), +-inf entries (NaN products ->
    INT32_MIN -> -128), values near FLT_MAX, negative zeros.  The fused
    preamble and the prep kernel must both reproduce the reference."""
    M, K, N = 8, 1024, 128
    rng = np.random.default_rng(5)
    x = rng.standard_normal((M, K)).astype(np.float32)
    x[0] = rng.standard_normal(K).astype(np.float32) * np.float32(1e-41)  # denormals
    x[1, 5], x[1, 77] = np.inf, -np.inf
    x[2] = rng.uniform(-3.4e38, 3.4e38, K).astype(np.float32)
    x[3] = -0.0
    x[4, 10] = 3e-39  # one denormal next to normal values
    bq, s4 = F.synth_q4g(N, K, 64, 9)
    for hsz in (0, 64):
        _, _, qs, pa = orc.prep_rows(x, M, K, hsz)
        c = torch.full((M, N), -5.0, device="cuda")
        fg.device.linear_q4g(D(x), K, hsz, M, N, K, D(bq), D(s4), 64, c)
        torch.cuda.synchronize()
        want = orc.gemm_q4g(M, N, K, pa, qs, bq, s4, 64)
        got = c.cpu().numpy()
        same = (got.view(np.uint32) == want.view(np.uint32)) | (np.isnan(got) & np.isnan(want))
        assert same.all(), f"hsz={hsz}: {int((~same).sum())} differ"


def test_linear_q8c_device_tensor_core_path(orc):
    """M >= 64 with a prepared weight: prep into temporary memory, then tcgen05."""
    M, K, N, hsz = 256, 2048, 512, 128
    x = np.random.default_rng(11).standard_normal((M, K)).astype(np.float32)
    _, _, qs, pa = orc.prep_rows(x, M, K, hsz)
    b8, s8 = F.synth_q8c(N, K, 17)
    bd = D(b8)
    fg.device.q8c_prepare(bd, N, K)
    try:
        c = torch.empty((M, N), device="cuda")
        fg.device.linear_q8c(D(x), K, hsz, M, N, K, bd, D(s8), c)
        torch.cuda.synchronize()
        assert_bits(c.cpu().numpy(), orc.gemm_q8c(M, N, K, pa, qs, b8, s8), "linear_q8c tc")
    finally:
        fg.device.q8c_release(bd)


@pytest.mark.parametrize("m,k,lda,hsz", [(1, 64, 64, 0), (7, 2048, 2100, 128), (16, 256, 256, 4),
                                         (20, 512, 512, 32), (256, 2048, 2048, 128),
                                         (3, 16384, 16384, 2048), (5, 3072, 3075, 1024),
                                         (9, 16384, 16384, 128), (2, 192, 192, 64),
                                         (4, 8192, 8192, 512), (33, 32768, 32768, 128)])
def test_prep_device_vs_oracle(orc, m, k, lda, hsz):
    x = np.random.default_rng(m + k + hsz).standard_normal((m, lda)).astype(np.float32) * 3
    rot, qa, qs, pa = orc.prep_rows(x, m, k, hsz, lda=lda)
    rd = torch.empty((m, k), device="cuda")
    qad = torch.empty((m, k), dtype=torch.int8, device="cuda")
    qsd = torch.empty(m, device="cuda")
    pad = torch.full((pa.size,), 99, dtype=torch.int8, device="cuda")
    fg.device.prep_rows(D(x), lda, qsd, pad, m, k, hsz, rot=rd, qa=qad)
    torch.cuda.synchronize()
    assert np.array_equal(rd.cpu().numpy().view(np.uint32), rot.view(np.uint32))
    assert np.array_equal(qad.cpu().numpy(), qa)
    assert np.array_equal(qsd.cpu().numpy().view(np.uint32), qs.view(np.uint32))
    assert np.array_equal(pad.cpu().numpy(), pa)


def test_fwht_and_quant_act_host_entries(orc):
    x = np.random.default_rng(3).standard_normal((4, 1024)).astype(np.float32)
    y = x.copy()
    fg.fwht(y, 128)
    assert np.array_equal(y.view(np.uint32), orc.fwht(x, 128).view(np.uint32))
    q = np.zeros((4, 1024), np.int8)
    s = np.zeros(4, np.float32)
    fg.quant_act(x, 4, 1024, q, s)
    q0, s0 = orc.quant_act(x)
    assert np.array_equal(q, q0) and np.array_equal(s.view(np.uint32), s0.view(np.uint32))


def test_registry_and_errors():
    from fastgemma_b200 import _lib
    L = _lib.lib()
    blob = np.arange(4096, dtype=np.uint8)
    before = L.fgm_cuda_registry_bytes()
    fg.register(blob)
    assert L.fgm_cuda_lookup(blob.ctypes.data)
    assert L.fgm_cuda_registry_bytes() == before + 4096
    assert L.fgm_cuda_register(blob.ctypes.data, 100) == -1  # size mismatch
    fg.unregister(blob)
    assert not L.fgm_cuda_lookup(blob.ctypes.data)
    with pytest.raises(fg.FgmCudaError):
        fg.unregister(blob)
    # device path rejects contract violations before launching
    c = torch.empty(64, device="cuda")
    assert L.fgm_cuda_gemm_q4g(8, 64, 100, c.data_ptr(), c.data_ptr(), c.data_ptr(),
                               c.data_ptr(), 64, c.data_ptr(), 64, 0, 4, None) == -1


def test_launch_counter_counts_kernels():
    from fastgemma_b200 import _lib
    L = _lib.lib()
    M, N, K = 2, 64, 128
    a = torch.zeros(16 * K, dtype=torch.int8, device="cuda")
    s = torch.ones(M, device="cuda")
    b = torch.zeros(N * K // 2, dtype=torch.uint8, device="cuda")
    bs = torch.zeros((K // 64) * N, dtype=torch.int16, device="cuda")
    c = torch.empty((M, N), device="cuda")
    n0 = L.fgm_cuda_launch_count()
    fg.device.gemm_q4g(M, N, K, a, s, b, bs, 64, c)
    torch.cuda.synchronize()
    assert L.fgm_cuda_launch_count() == n0 + 1


# ------------------------------------------- prefill: tcgen05 tensor-core path
@pytest.mark.parametrize("M,K,N,n0,n1,cpad", [(64, 1024, 256, 0, 16, 16), (100, 2048, 512, 4, 24, 16),
                                             (256, 2048, 512, 0, 32, 16), (256, 8192, 256, 0, 16, 16),
                                             (300, 2048, 384, 0, 24, 16), (1024, 2048, 256, 8, 16, 16),
                                             (256, 8192, 256, 4, 12, 3), (130, 4096, 1024, 0, 64, 5),
                                             (256, 16384, 2048, 0, 128, 16),
                                             (256, 2048, 6144, 0, 384, 16),
                                             # more 128 x 256 tiles than SMs: the persistent
                                             # kernel (153 tiles, the last 192 columns wide;
                                             # 150 tiles from n-block 8)
                                             (384, 512, 12992, 0, 812, 16),
                                             (200, 768, 19456, 8, 1208, 4)])
def test_q8c_tensor_core_bit_exact(orc, M, K, N, n0, n1, cpad):
    """M >= 64 with a prepared weight runs tcgen05.mma kind::i8 (K split over a
    cluster when the output has few tiles, one persistent CTA per SM with two
    tensor-memory accumulators when it has many); f32 outputs and int32
    accumulators must match the reference arithmetic exactly, with aligned
    and unaligned output rows (ldc = N + cpad)."""
    rng = np.random.default_rng(M * 31 + K + N)
    A = rng.integers(-128, 128, size=(M, K), dtype=np.int8)
    b, s = F.synth_q8c(N, K, M + 7 * N)
    a_s = rng.uniform(0.001, 0.05, size=M).astype(np.float32)
    pa = F.pack_a(A)
    pad, bd, sd, asd = D(pa), D(b), D(s), D(a_s)
    fg.device.q8c_prepare(bd, N, K)
    try:
        ldc = N + cpad
        c = torch.full((M, ldc), -9.0, device="cuda")
        fg.device.gemm_q8c(M, N, K, pad, asd, bd, sd, c, ldc, n0, n1)
        acc = torch.full((M, N), 7, dtype=torch.int32, device="cuda")
        fg.device.gemm_q8c_acc(M, N, K, pad, bd, acc, n0, n1)
        torch.cuda.synchronize()
        from fastgemma_b200 import _lib
        assert _lib.lib().fgm_cuda_device_status() == 0
        want = np.full((M, ldc), -9.0, np.float32)
        orc.gemm_q8c(M, N, K, pa, a_s, b, s, c=want, ldc=ldc, n0=n0, n1=n1)
        assert_bits(c.cpu().numpy(), want, f"tc q8c M={M} K={K} N={N}")
        want_acc = orc.gemm_q8c_acc(M, N, K, pa, b, n0, n1)
        got_acc = acc.cpu().numpy()
        cols = slice(n0 * 16, n1 * 16)
        assert np.array_equal(got_acc[:, cols], want_acc[:, cols])
    finally:
        fg.device.q8c_release(bd)


def test_q8c_prefill_config2_sampled(orc):
    """BASELINE config 2 at full size (M=256, K=2048, N=16384) on the tensor
    cores: column blocks across the width checked against the oracle, and the
    GPU's own two paths (tensor core vs streaming kernel) agree everywhere."""
    M, K, N = 256, 2048, 16384
    x = F.synth_x(M, K, 5)
    b, s = F.synth_q8c(N, K, 6, structured=False)
    _, _, qs, pa = orc.prep_rows(x, M, K, 0)
    pad, bd, sd, qsd = D(pa), D(b), D(s), D(qs)
    c_mma = torch.empty((M, N), device="cuda")
    fg.device.gemm_q8c(M, N, K, pad, qsd, bd, sd, c_mma)  # not prepared: streaming kernel
    fg.device.q8c_prepare(bd, N, K)
    try:
        c_tc = torch.empty((M, N), device="cuda")
        fg.device.gemm_q8c(M, N, K, pad, qsd, bd, sd, c_tc)
        torch.cuda.synchronize()
        got = c_tc.cpu().numpy()
        assert np.array_equal(got.view(np.uint32), c_mma.cpu().numpy().view(np.uint32))
        for a in (0, 252, 512, 1020):
            want = np.zeros((M, N), np.float32)
            orc.gemm_q8c(M, N, K, pa, qs, b, s, c=want, n0=a, n1=a + 4)
            assert_bits(got[:, a * 16:(a + 4) * 16], want[:, a * 16:(a + 4) * 16], f"nb {a}")
    finally:
        fg.device.q8c_release(bd)


def test_q8c_host_path_prepares_registered_weights(orc):
    """The host-pointer drop-in with a registered int8 weight at M >= 64 goes
    through the tensor cores (prepared on first use) and stays bit-exact."""
    M, K, N = 128, 2048, 256
    rng = np.random.default_rng(17)
    A = rng.integers(-128, 128, size=(M, K), dtype=np.int8)
    b, s = F.synth_q8c(N, K, 18)
    a_s = rng.uniform(0.001, 0.05, size=M).astype(np.float32)
    pa = F.pack_a(A)
    fg.register(b)
    try:
        c = np.zeros((M, N), np.float32)
        fg.gemm_q8c(M, N, K, pa, a_s, b, s, c, N, 0, N // 16)
        assert_bits(c, orc.gemm_q8c(M, N, K, pa, a_s, b, s), "host tc")
    finally:
        fg.unregister(b)


@pytest.mark.parametrize("M,K,N", [(256, 2048, 1024), (77, 1024, 256), (512, 8192, 128)])
def test_q8c_rows_entry_from_quantiser(orc, M, K, N):
    """Prefill form: quantise on the device (row-major int8 out), then the
    tensor-core GEMM straight from it; equals prep + reference GEMM."""
    x = F.synth_x(M, K, M + K + N)
    b, s = F.synth_q8c(N, K, N + 3)
    _, qa, qs, pa = orc.prep_rows(x, M, K, 128)
    xd, bd, sd = D(x), D(b), D(s)
    qad = torch.empty((M, K), dtype=torch.int8, device="cuda")
    qsd = torch.empty(M, device="cuda")
    pad = torch.empty(pa.size, dtype=torch.int8, device="cuda")
    fg.device.prep_rows(xd, K, qsd, pad, M, K, 128, qa=qad)
    fg.device.q8c_prepare(bd, N, K)
    try:
        c = torch.empty((M, N), device="cuda")
        fg.device.gemm_q8c_rows(M, N, K, qad, qsd, bd, sd, c)
        torch.cuda.synchronize()
        assert np.array_equal(qad.cpu().numpy(), qa)
        assert_bits(c.cpu().numpy(), orc.gemm_q8c(M, N, K, pa, qs, b, s), f"rows M={M}")
    finally:
        fg.device.q8c_release(bd)
    with pytest.raises(fg.FgmCudaError):  # unprepared weights are refused, not computed slowly
        fg.device.gemm_q8c_rows(M, N, K, qad, qsd, bd, sd, c)


# ------------------------------------------------ column-sharded large-N GEMM
@pytest.mark.parametrize("kind,world", [("q4g", 1), ("q4g", 2), ("q4g", 8), ("q8c", 3)])
def test_column_shards_on_device_assemble_to_the_whole_gemm(orc, kind, world):
    """Every rank's shard (the LM-head split) run on one device and assembled
    equals the unsplit GEMM bit for bit."""
    from fastgemma_b200 import shard as S
    M, N, K = 8, 4096, 2048
    if kind == "q4g":
        blob, scale = F.synth_q4g(N, K, 64, 21, structured=False)
    else:
        blob, scale = F.synth_q8c(N, K, 21, structured=False)
    rng = np.random.default_rng(4)
    pa = F.pack_a(rng.integers(-128, 128, size=(M, K), dtype=np.int8))
    a_s = rng.uniform(0.01, 0.1, size=M).astype(np.float32)
    shards = [S.ColumnShardedGemm(kind, blob, scale, N, K, 64, rank=r, world=world, device="cuda")
              for r in range(world)]
    blocks = torch.stack([sh.local(M, D(pa), D(a_s)).clone() for sh in shards])
    out = S.assemble(blocks, shards[0].ranges, torch.empty((M, N), device="cuda"))
    torch.cuda.synchronize()
    want = (orc.gemm_q4g(M, N, K, pa, a_s, blob, scale, 64) if kind == "q4g"
            else orc.gemm_q8c(M, N, K, pa, a_s, blob, scale))
    assert_bits(out.cpu().numpy(), want, f"{kind} world={world}")


def test_fused_gather_single_rank_calls(orc):
    """The fused GEMM + gather kernel at world size 1 (its own buffer and
    counters): several calls alternate the double buffers and each result
    matches the oracle."""
    from fastgemma_b200 import shard as S
    M, N, K = 8, 2048, 2048
    blob, scale = F.synth_q4g(N, K, 64, 91, structured=False)
    sh = S.ColumnShardedGemm("q4g", blob, scale, N, K, 64, rank=0, world=1, device="cuda",
                             fused=True)
    try:
        rng = np.random.default_rng(9)
        outs = []
        for i in range(4):
            A = rng.integers(-128, 128, size=(M, K), dtype=np.int8)
            a_s = rng.uniform(0.01, 0.1, size=M).astype(np.float32)
            pa = F.pack_a(A)
            got = sh.fused_call(M, D(pa), D(a_s))
            torch.cuda.synchronize()
            from fastgemma_b200 import _lib
            assert _lib.lib().fgm_cuda_device_status() == 0
            assert_bits(got.cpu().numpy(), orc.gemm_q4g(M, N, K, pa, a_s, blob, scale, 64),
                        f"call {i}")
            outs.append(got)
        assert outs[0].data_ptr() == outs[2].data_ptr() != outs[1].data_ptr()
    finally:
        sh.close()


@pytest.mark.parametrize("M,N,col0", [(8, 262144, 0), (3, 5000, 16), (16, 8192, 0), (1, 64, 128)])
def test_argmax_partials_and_merge_match_the_reference_scan(orc, M, N, col0):
    """Row argmax (engine.rs:75-83) from chunk partials: ties keep the first
    index, NaN never wins, an all -inf / NaN row answers 0."""
    from fastgemma_b200 import _lib
    L = _lib.lib()
    rng = np.random.default_rng(N + M)
    c = rng.standard_normal((M, N)).astype(np.float32)
    if M > 2:
        c[1, :] = -np.inf
        c[1, 7] = np.nan  # nothing above -inf: 0
        c[2, N // 3] = c[2, N - 5] = 99.0  # a tie: the earlier one
        c[2, N // 2] = np.nan
    if M > 5:
        c[5, :] = c[5, 11]  # all equal: index 11's value first occurs at 0
        c[5, 0] = c[5, 11] - 1
    parts = L.fgm_cuda_argmax_parts(N)
    cd = D(c)
    vals = torch.empty((M, parts), device="cuda")
    idx = torch.empty((M, parts), dtype=torch.int32, device="cuda")
    out = torch.empty(M, dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    _lib.call("fgm_cuda_argmax_partials", cd.data_ptr(), M, N, N, col0, vals.data_ptr(),
              idx.data_ptr(), s)
    _lib.call("fgm_cuda_argmax_merge", vals.data_ptr(), idx.data_ptr(), M, parts, out.data_ptr(), s)
    torch.cuda.synchronize()
    want = orc.argmax_rows(c)
    got = out.cpu().numpy()
    offset = np.where(np.isin(np.arange(M), [1] if M > 2 else []), 0, col0)
    assert np.array_equal(got, want + offset), (got, want)


@pytest.mark.parametrize("world", [1, 2, 8])
def test_sharded_lm_head_argmax_equals_argmax_of_whole_logits(orc, world):
    """Every rank's shard reduced to (value, index) pairs and merged (the
    exchange emulated on one device) picks the token the reference picks from
    the whole logits."""
    from fastgemma_b200 import _lib
    from fastgemma_b200 import shard as S
    M, N, K = 8, 16384, 2048
    blob, scale = F.synth_q4g(N, K, 64, 55, structured=False)
    rng = np.random.default_rng(12)
    pa = F.pack_a(rng.integers(-128, 128, size=(M, K), dtype=np.int8))
    a_s = rng.uniform(0.01, 0.1, size=M).astype(np.float32)
    shards = [S.ColumnShardedGemm("q4g", blob, scale, N, K, 64, rank=r, world=world,
                                  device="cuda") for r in range(world)]
    L = _lib.lib()
    s = torch.cuda.current_stream().cuda_stream
    parts = L.fgm_cuda_argmax_parts(shards[0].max_cols)
    vs, ids = [], []
    for sh in shards:
        loc = sh.local(M, D(pa), D(a_s))
        v = torch.empty((M, parts), device="cuda")
        i = torch.empty((M, parts), dtype=torch.int32, device="cuda")
        _lib.call("fgm_cuda_argmax_partials", loc.data_ptr(), M, sh.cols, sh.max_cols,
                  sh.nb0 * 16, v.data_ptr(), i.data_ptr(), s)
        vs.append(v.clone())
        ids.append(i.clone())
    vals = torch.cat(vs, 1).contiguous()
    idx = torch.cat(ids, 1).contiguous()
    out = torch.empty(M, dtype=torch.int32, device="cuda")
    _lib.call("fgm_cuda_argmax_merge", vals.data_ptr(), idx.data_ptr(), M, vals.shape[1],
              out.data_ptr(), s)
    torch.cuda.synchronize()
    logits = orc.gemm_q4g(M, N, K, pa, a_s, blob, scale, 64)
    assert np.array_equal(out.cpu().numpy(), orc.argmax_rows(logits))
    if world == 1:
        assert np.array_equal(shards[0].argmax(M, D(pa), D(a_s)).cpu().numpy(),
                              orc.argmax_rows(logits))
