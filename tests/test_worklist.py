"""The decode work list (fgm_cuda_worklist_*): many preps and decode GEMMs in
one persistent launch.  Every output must equal the per-call entries' -- and
so the oracle's -- bit for bit: preps against orc.prep_rows, int4 GEMMs
against orc.gemm_q4g, int8 GEMMs against orc.gemm_q8c, including entries that
read another entry's output inside the same launch (a GEMM, the prep of its
output, the next GEMM: forward.rs:128-158 twice), column ranges, ldc > N, and
repeated runs of one list (the counters reset between runs)."""
import ctypes as C

import numpy as np
import pytest

from fastgemma_b200 import _lib
from fastgemma_b200 import fgm_format as F

torch = pytest.importorskip("torch")
import fastgemma_b200.device as D  # noqa: E402


def _work(**kw):
    w = D._Work(**{k: v for k, v in kw.items() if k != "deps"})
    d = list(kw.get("deps", ())) + [-1, -1]
    w.deps[0], w.deps[1] = d[0], d[1]
    return w


def _create(M, works):
    arr = (D._Work * len(works))(*works)
    h = C.c_void_p()
    rc = _lib.lib().fgm_cuda_worklist_create(M, arr, len(works), C.byref(h))
    return rc, _lib.lib().fgm_cuda_last_error().decode()


P = 1 << 12  # a fake, aligned, never-dereferenced address (validation comes first)


@pytest.mark.parametrize("M,work,why", [
    (0, dict(kind=2, K=128, lda=128, src=P, pa=P, qs=P), "M=0"),
    (17, dict(kind=2, K=128, lda=128, src=P, pa=P, qs=P), "M=17"),
    (8, dict(kind=2, K=96, lda=96, src=P, pa=P, qs=P), "K %% 128"),
    (8, dict(kind=2, K=128, lda=128, hsz=256, src=P, pa=P, qs=P), "hsz"),
    (8, dict(kind=2, K=128, lda=130, src=P, pa=P, qs=P), "lda"),
    (8, dict(kind=2, K=128, lda=128, src=P + 4, pa=P, qs=P), "aligned"),
    (8, dict(kind=0, N=64, K=1024, group=64, n0=0, n1=4, ldc=64, A=P, a_scale=P, B=P, b_scale=P,
             C=P, deps=(0,)), "dependency"),
    (8, dict(kind=0, N=64, K=768, group=64, n0=0, n1=4, ldc=64, A=P, a_scale=P, B=P, b_scale=P,
             C=P), "K %% 512"),
    (8, dict(kind=0, N=64, K=1024, group=1024, n0=0, n1=4, ldc=64, A=P, a_scale=P, B=P,
             b_scale=P, C=P), "group"),
    (8, dict(kind=1, N=64, K=512, n0=2, n1=2, ldc=64, A=P, a_scale=P, B=P, b_scale=P, C=P),
     "n-blocks"),
    (8, dict(kind=1, N=64, K=512, n0=0, n1=4, ldc=48, A=P, a_scale=P, B=P, b_scale=P, C=P),
     "ldc"),
    (8, dict(kind=1, N=64, K=512, n0=0, n1=4, ldc=64, A=P + 8, a_scale=P, B=P, b_scale=P, C=P),
     "aligned"),
    (8, dict(kind=1, N=64, K=512, n0=0, n1=4, ldc=64, A=P, a_scale=0, B=P, b_scale=P, C=P),
     "null"),
    (8, dict(kind=5, N=64, K=512, n0=0, n1=4, ldc=64), "kind"),
])
def test_worklist_rejects_out_of_contract_entries(M, work, why):
    rc, msg = _create(M, [_work(**work)])
    assert rc == -1, msg
    assert why.replace("%%", "%") in msg, msg


def _gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)


def Dv(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def bits_equal(got, want):
    got, want = np.asarray(got, np.float32), np.asarray(want, np.float32)
    same = got.view(np.uint32) == want.view(np.uint32)
    return bool(same.all()), int((~same).sum())


@pytest.mark.gpu
@pytest.mark.parametrize("M", [1, 3, 8, 9, 16])
def test_config1_layers_in_one_launch(orc, M):
    """Two layers of the config-1 projections (q, kv, o, gate/up, down; int4
    g64) with their four preps each, as one list: preps first, every GEMM
    waiting on its prep inside the launch."""
    _gpu()
    shapes = [("q", 2048, 2048, 0), ("kv", 2048, 512, 0), ("o", 2048, 2048, 1),
              ("gate_up", 2048, 4096, 2), ("down", 8192, 2048, 3)]
    rng = np.random.default_rng(100 + M)
    wl = D.WorkList()
    host, dev_out = [], []
    for layer in range(2):
        xs = [rng.standard_normal((M, K), dtype=np.float32) for K in (2048, 2048, 2048, 8192)]
        preps = []
        for x in xs:
            K = x.shape[1]
            xd, pa = Dv(x), D.packed_a(M, K)
            qs = torch.empty(M, device="cuda")
            preps.append((wl.prep(xd, K, K, pa, qs), pa, qs))
        for name, K, N, inp in shapes:
            bq, s = F.synth_q4g(N, K, 64, 7 * layer + N + K, structured=False)
            c = torch.full((M, N), -1.0, device="cuda")
            idx, pa, qs = preps[inp]
            wl.gemm_q4g(N, K, pa, qs, Dv(bq), Dv(s.view(np.uint16)), 64, c, deps=(idx,))
            host.append((xs[inp], bq, s, N, K))
            dev_out.append(c)
    wl.build(M)
    for _ in range(2):  # the second run finds the counters reset
        for c in dev_out:
            c.fill_(-1.0)
        wl.run()
        torch.cuda.synchronize()
        assert _lib.lib().fgm_cuda_device_status() == 0
        for (x, bq, s, N, K), c in zip(host, dev_out):
            _, _, qs_r, pa_r = orc.prep_rows(x, M, K, 0)
            want = orc.gemm_q4g(M, N, K, pa_r, qs_r, bq, s, 64)[:M]
            ok, nd = bits_equal(c.cpu().numpy(), want)
            assert ok, f"N={N} K={K}: {nd} outputs differ"
    wl.close()


def _rows(pa, K, M):
    """Rows [0, M) of a tile-packed 16-row block [K/64][16][64]."""
    return pa.reshape(K // 64, 16, 64)[:, :M, :]


@pytest.mark.gpu
@pytest.mark.parametrize("M,hsz", [(8, 0), (8, 128), (16, 64), (5, 128)])
def test_chain_gemm_prep_gemm_inside_one_launch(orc, M, hsz):
    """x -> prep -> int4 GEMM (N1) -> prep of its output -> int8 GEMM, plus an
    int4 GEMM with group 256 over a column range and ldc > N -- every
    dependency resolved by counters in the same launch; the preps' packed
    rows and scales are checked too."""
    _gpu()
    rng = np.random.default_rng(7 * M + hsz)
    K1, N1, N2, N3 = 2048, 1024, 512, 768
    x = rng.standard_normal((M, K1), dtype=np.float32)
    b1, s1 = F.synth_q4g(N1, K1, 64, 1, structured=False)
    b2, s2 = F.synth_q8c(N2, N1, 2, structured=False)
    b3, s3 = F.synth_q4g(N3, K1, 256, 3, structured=False)
    xd = Dv(x)
    pa1, qs1 = D.packed_a(M, K1), torch.empty(M, device="cuda")
    pa2, qs2 = D.packed_a(M, N1), torch.empty(M, device="cuda")
    c1 = torch.full((M, N1), 5.0, device="cuda")
    c2 = torch.full((M, N2), 5.0, device="cuda")
    ldc3 = N3 + 32
    c3 = torch.full((M, ldc3), 5.0, device="cuda")
    wl = D.WorkList()
    i0 = wl.prep(xd, K1, K1, pa1, qs1, hsz=hsz)
    i1 = wl.gemm_q4g(N1, K1, pa1, qs1, Dv(b1), Dv(s1.view(np.uint16)), 64, c1, deps=(i0,))
    i2 = wl.prep(c1, N1, N1, pa2, qs2, hsz=hsz, deps=(i1,))
    wl.gemm_q8c(N2, N1, pa2, qs2, Dv(b2), Dv(s2), c2, deps=(i2,))
    wl.gemm_q4g(N3, K1, pa1, qs1, Dv(b3), Dv(s3.view(np.uint16)), 256, c3, ldc=ldc3, n0=4, n1=40,
                deps=(i0,))
    wl.build(M)
    for _ in range(3):
        wl.run()
    torch.cuda.synchronize()
    assert _lib.lib().fgm_cuda_device_status() == 0
    _, _, qs1_r, pa1_r = orc.prep_rows(x, M, K1, hsz)
    # rows [0, M) of the packed block (a prep that depends on no entry leaves
    # the padding rows as they are)
    assert np.array_equal(_rows(pa1.cpu().numpy(), K1, M), _rows(pa1_r, K1, M))
    assert np.array_equal(qs1.cpu().numpy().view(np.uint32), qs1_r.view(np.uint32))
    want1 = orc.gemm_q4g(M, N1, K1, pa1_r, qs1_r, b1, s1, 64)[:M]
    assert bits_equal(c1.cpu().numpy(), want1)[0]
    _, _, qs2_r, pa2_r = orc.prep_rows(want1, M, N1, hsz)
    assert np.array_equal(pa2.cpu().numpy(), pa2_r)
    want2 = orc.gemm_q8c(M, N2, N1, pa2_r, qs2_r, b2, s2)[:M]
    assert bits_equal(c2.cpu().numpy(), want2)[0]
    want3 = np.full((M, ldc3), 5.0, np.float32)
    orc.gemm_q4g(M, N3, K1, pa1_r, qs1_r, b3, s3, 256, c=want3, ldc=ldc3, n0=4, n1=40)
    assert bits_equal(c3.cpu().numpy(), want3)[0]
    wl.close()


@pytest.mark.gpu
def test_worklist_matches_the_per_call_kernels_at_full_config1_width(orc):
    """One full config-1 layer at M = 8 (gate/up at its 16384 width), list vs
    the per-call entries (prep_rows + gemm_q4g): identical bits."""
    _gpu()
    M = 8
    shapes = [(2048, 2048), (2048, 512), (2048, 2048), (2048, 16384), (8192, 2048)]
    rng = np.random.default_rng(5)
    wl = D.WorkList()
    outs = []
    gen = torch.Generator(device="cuda")
    gen.manual_seed(11)
    for K, N in shapes:
        x = torch.randn((M, K), device="cuda", generator=gen)
        pa, qs = D.packed_a(M, K), torch.empty(M, device="cuda")
        w = torch.randint(0, 256, (N * K // 2,), dtype=torch.uint8, device="cuda", generator=gen)
        s = torch.empty((K // 64, N), device="cuda").uniform_(0.005, 0.02, generator=gen).half()
        c = torch.empty((M, N), device="cuda")
        ip = wl.prep(x, K, K, pa, qs)
        wl.gemm_q4g(N, K, pa, qs, w, s, 64, c, deps=(ip,))
        outs.append((x, w, s, c, K, N))
    wl.build(M)
    wl.run()
    torch.cuda.synchronize()
    for x, w, s, c, K, N in outs:
        pa, qs = D.packed_a(M, K), torch.empty(M, device="cuda")
        ref = torch.empty((M, N), device="cuda")
        D.prep_rows(x, K, qs, pa, M, K, 0)
        D.gemm_q4g(M, N, K, pa, qs, w, s, 64, ref)
        torch.cuda.synchronize()
        assert torch.equal(ref.view(torch.int32), c.view(torch.int32)), f"K={K} N={N}"
    assert _lib.lib().fgm_cuda_device_status() == 0
    wl.close()
    del rng


@pytest.mark.gpu
def test_many_long_dependency_free_preps(orc):
    """24 preps of K = 16384 that depend on nothing (192 rows over the CTAs:
    some CTAs prepare two rows, more chunks per warp than one held batch, so
    the second pass reloads), a third of them with the FWHT, each feeding an
    int4 GEMM.  Outputs, packed rows [0, M) and scales against the oracle,
    bit for bit."""
    _gpu()
    M, K, N, P = 8, 16384, 64, 24
    rng = np.random.default_rng(41)
    xs = [rng.standard_normal((M, K), dtype=np.float32) * (1 + i) for i in range(P)]
    b, s = F.synth_q4g(N, K, 64, 9, structured=False)
    bd, sd = Dv(b), Dv(s.view(np.uint16))
    wl = D.WorkList()
    outs = []
    for i, x in enumerate(xs):
        pa, qs = D.packed_a(M, K), torch.empty(M, device="cuda")
        ip = wl.prep(Dv(x), K, K, pa, qs, hsz=128 if i % 3 == 0 else 0)
        c = torch.empty((M, N), device="cuda")
        wl.gemm_q4g(N, K, pa, qs, bd, sd, 64, c, deps=(ip,))
        outs.append((pa, qs, c))
    wl.build(M)
    for _ in range(2):
        wl.run()
    torch.cuda.synchronize()
    assert _lib.lib().fgm_cuda_device_status() == 0
    for i, (x, (pa, qs, c)) in enumerate(zip(xs, outs)):
        hsz = 128 if i % 3 == 0 else 0
        _, _, qs_r, pa_r = orc.prep_rows(x, M, K, hsz)
        assert np.array_equal(_rows(pa.cpu().numpy(), K, M), _rows(pa_r, K, M)), i
        assert np.array_equal(qs.cpu().numpy().view(np.uint32), qs_r.view(np.uint32)), i
        want = orc.gemm_q4g(M, N, K, pa_r, qs_r, b, s, 64)[:M]
        assert bits_equal(c.cpu().numpy(), want)[0], i
    wl.close()


@pytest.mark.gpu
def test_host_inputs_and_outputs(orc):
    """Prep sources and GEMM outputs in page-locked host memory (the kernel
    reads and writes them through their device mapping): bit for bit the
    oracle's results, on two runs; a pageable host buffer is rejected."""
    _gpu()
    M, K, N = 8, 2048, 512
    rng = np.random.default_rng(23)
    x = rng.standard_normal((M, K), dtype=np.float32)
    b, s = F.synth_q4g(N, K, 64, 4, structured=False)
    xh = torch.from_numpy(x).pin_memory()
    ch = torch.zeros((M, N), dtype=torch.float32).pin_memory()
    pa, qs = D.packed_a(M, K), torch.empty(M, device="cuda")
    wl = D.WorkList()
    ip = wl.prep(xh, K, K, pa, qs)
    wl.gemm_q4g(N, K, pa, qs, Dv(b), Dv(s.view(np.uint16)), 64, ch, deps=(ip,))
    wl.build(M)
    _, _, qs_r, pa_r = orc.prep_rows(x, M, K, 0)
    want = orc.gemm_q4g(M, N, K, pa_r, qs_r, b, s, 64)[:M]
    for _ in range(2):
        ch.zero_()
        wl.run()
        torch.cuda.synchronize()
        assert _lib.lib().fgm_cuda_device_status() == 0
        assert bits_equal(ch.numpy(), want)[0]
    wl.close()
    # pageable host memory cannot be reached by the kernel: rejected at creation
    cp = torch.zeros((M, N), dtype=torch.float32)
    bad = D.WorkList()
    bad.gemm_q4g(N, K, pa, qs, Dv(b), Dv(s.view(np.uint16)), 64, cp)
    with pytest.raises(_lib.FgmCudaError):
        bad.build(M)
