"""The decode-chain glue and the int8-KV attention on the device
(csrc/glue.cu) against the oracle's restatement of ops.c, itself pinned
bit-exact against the reference kernels (tests/test_oracle.py).  Row lengths
that are multiples of 16 must match bit for bit; the reference's libm pieces
(scalar tails, rope, the softmax tail) are compared to REL_TOL."""
import numpy as np
import pytest

import fastgemma_b200.device as D

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
REL_TOL, ABS_TOL = 2e-6, 1e-6


@pytest.fixture(scope="module", autouse=True)
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def same(got, want, exact, what):
    got, want = np.asarray(got, np.float32), np.asarray(want, np.float32)
    if exact:
        bad = got.view(np.uint32) != want.view(np.uint32)
        assert not bad.any(), f"{what}: {int(bad.sum())} differ, e.g. {got[bad][:3]} vs {want[bad][:3]}"
    else:
        assert np.allclose(got, want, rtol=REL_TOL, atol=ABS_TOL), \
            f"{what}: max abs {np.abs(got - want).max()}"


@pytest.mark.parametrize("n", [16, 2048, 8192, 2056])
def test_rmsnorm_gelu_softcap_elementwise(orc, n):
    rng = np.random.default_rng(n)
    rows = 5
    x = (rng.standard_normal((rows, n)) * 3).astype(np.float32)
    w = rng.standard_normal(n).astype(np.float32)
    exact = n % 16 == 0
    for wt in (w, None):
        out = torch.empty((rows, n), device="cuda")
        D.rmsnorm(out, dev(x), None if wt is None else dev(wt), rows, n, 1e-6)
        torch.cuda.synchronize()
        same(out.cpu().numpy(), orc.rmsnorm(x, wt, 1e-6), exact, f"rmsnorm n={n}")
    g = (rng.standard_normal((rows, n)) * 4).astype(np.float32)
    u = rng.standard_normal((rows, n)).astype(np.float32)
    out = torch.empty((rows, n), device="cuda")
    D.gelu_mul(out, dev(g), dev(u), rows, n)
    torch.cuda.synchronize()
    want = np.stack([orc.gelu_mul(g[r], u[r]) for r in range(rows)])
    same(out.cpu().numpy(), want, exact, f"gelu_mul n={n}")
    xc = dev(g * 10)
    D.softcap(xc, rows, n, 30.0)
    torch.cuda.synchronize()
    want = np.stack([orc.softcap(g[r] * 10, 30.0) for r in range(rows)])
    same(xc.cpu().numpy(), want, exact, f"softcap n={n}")
    a = dev(g)
    D.add(a, dev(u))
    D.mul(a, dev(u))
    D.scale(a, 0.375)
    torch.cuda.synchronize()
    same(a.cpu().numpy(), ((g + u) * u) * np.float32(0.375), True, "add/mul/scale")


def test_rope_rows_with_their_positions(orc):
    rng = np.random.default_rng(3)
    rows, nh, hd = 4, 8, 256
    inv = (1.0 / (10000 ** (np.arange(0, hd, 2) / hd))).astype(np.float32)
    inv[-16:] = 0.0
    x = rng.standard_normal((rows, nh * hd)).astype(np.float32)
    pos = np.array([0, 7, 513, 4095], np.int32)
    xd = dev(x)
    D.rope(xd, nh * hd, rows, nh, hd, dev(inv), dev(pos))
    torch.cuda.synchronize()
    want = np.stack([orc.rope(x[r], nh, hd, inv, int(pos[r])) for r in range(rows)])
    same(xd.cpu().numpy(), want, False, "rope")
    # with the host's libm table: bit for bit (position 4095 lies outside the
    # table and takes the device evaluation)
    cs = dev(D.rope_table(1024, hd, inv))
    xd = dev(x)
    D.rope(xd, nh * hd, rows, nh, hd, dev(inv), dev(pos), cs=cs)
    torch.cuda.synchronize()
    got = xd.cpu().numpy()
    same(got[:3], want[:3], True, "rope with the cos / sin table")
    same(got[3:], want[3:], False, "rope past the table")


def test_quant_act_and_store_v_t(orc):
    rng = np.random.default_rng(4)
    rows, k = 3, 512
    x = rng.standard_normal((rows, k)).astype(np.float32)
    x[1, :] = 0.0
    q = torch.empty((rows, k), dtype=torch.int8, device="cuda")
    s = torch.empty(rows, device="cuda")
    D.quant_act(dev(x), rows, k, q, s)
    torch.cuda.synchronize()
    wq, ws = orc.quant_act(x)
    assert np.array_equal(q.cpu().numpy(), wq)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), ws.view(np.uint32))
    cap, n = 10, 512
    vt = torch.zeros((rows, (cap + 2) * n), dtype=torch.int8, device="cuda")
    want = np.zeros((rows, (cap + 2) * n), np.int8)
    for slot in (0, 3, 4, 9):
        src = rng.integers(-127, 128, (rows, n)).astype(np.int8)
        D.store_v_t(vt, (cap + 2) * n, dev(src), n, rows, n, slot)
        for r in range(rows):
            orc.store_v_t(want[r], src[r], slot)
    torch.cuda.synchronize()
    assert np.array_equal(vt.cpu().numpy(), want)


def _caches(orc, rng, rows, cap, kvh, hd):
    kc = rng.integers(-127, 128, (rows, cap, kvh * hd)).astype(np.int8)
    ks = rng.uniform(0.001, 0.02, (rows, cap)).astype(np.float32)
    vslots = (cap + 3) // 4 * 4
    vt = np.zeros((rows, vslots * kvh * hd), np.int8)
    for r in range(rows):
        for sl in range(cap):
            orc.store_v_t(vt[r], rng.integers(-127, 128, kvh * hd).astype(np.int8), sl)
    vs = rng.uniform(0.001, 0.02, (rows, cap)).astype(np.float32)
    return kc, ks, vt, vs


@pytest.mark.parametrize("end,start,ring,hd", [(64, 0, 0, 256), (1024, 0, 0, 256),
                                               (1024, 16, 0, 512), (100, 0, 0, 256),
                                               (300, 41, 0, 128), (600, 500, 128, 256),
                                               (257, 129, 128, 256)])
def test_attention_rows_against_oracle(orc, end, start, ring, hd):
    """Three query rows, each with its own cache; 8 heads over 2 KV heads.
    Windows whose length is a multiple of 16 are bit-exact; others differ
    only through the softmax tail's exp (libm in the reference)."""
    rng = np.random.default_rng(end * 7 + start + ring + hd)
    rows, nh, kvh = 3, 8, 2
    cap = ring or end
    kc, ks, vt, vs = _caches(orc, rng, rows, cap, kvh, hd)
    q = (rng.standard_normal((rows, nh * hd)) * 2).astype(np.float32)
    out = torch.full((rows, nh * hd), float("nan"), device="cuda")
    D.attend_q8(out, nh * hd, dev(q), nh * hd, dev(kc), cap * kvh * hd, dev(ks), cap, dev(vt),
                vt.shape[1], dev(vs), cap, rows, nh, kvh, hd, start, end, ring)
    torch.cuda.synchronize()
    want = np.stack([orc.attend_q8(q[r], kc[r], ks[r], vt[r], vs[r], nh, kvh, hd, start, end, ring)
                     for r in range(rows)])
    same(out.cpu().numpy(), want, (end - start) % 16 == 0, f"attend [{start},{end}) ring={ring}")


@pytest.mark.parametrize("nh,kvh,hd,end,start,ring", [(2, 2, 256, 300, 0, 0), (8, 1, 128, 520, 7, 0),
                                                      (6, 2, 192, 200, 0, 0), (16, 1, 64, 96, 0, 0),
                                                      (8, 2, 512, 8192, 0, 0),
                                                      (4, 2, 256, 1100, 900, 512)])
def test_attention_head_groups_and_long_windows(orc, nh, kvh, hd, end, start, ring):
    """Query heads per KV head 1, 8, 3 and 16, and windows long enough to
    stream the K and V caches through several shared-memory stages."""
    rng = np.random.default_rng(nh * 131 + hd + end)
    rows = 2
    cap = ring or end
    kc, ks, vt, vs = _caches(orc, rng, rows, cap, kvh, hd)
    q = (rng.standard_normal((rows, nh * hd)) * 2).astype(np.float32)
    out = torch.full((rows, nh * hd), float("nan"), device="cuda")
    D.attend_q8(out, nh * hd, dev(q), nh * hd, dev(kc), cap * kvh * hd, dev(ks), cap, dev(vt),
                vt.shape[1], dev(vs), cap, rows, nh, kvh, hd, start, end, ring)
    torch.cuda.synchronize()
    want = np.stack([orc.attend_q8(q[r], kc[r], ks[r], vt[r], vs[r], nh, kvh, hd, start, end, ring)
                     for r in range(rows)])
    same(out.cpu().numpy(), want, (end - start) % 16 == 0, f"attend G={nh // kvh} hd={hd}")


def test_attention_caches_on_4_byte_boundaries(orc):
    """K and V caches that start 4 bytes past a 16-byte boundary take the
    4-byte copy path and give the same bits."""
    rng = np.random.default_rng(7)
    rows, nh, kvh, hd, n = 2, 8, 2, 256, 160
    kc, ks, vt, vs = _caches(orc, rng, rows, n, kvh, hd)
    kbuf = torch.zeros(kc.size + 16, dtype=torch.int8, device="cuda")
    vbuf = torch.zeros(vt.size + 16, dtype=torch.int8, device="cuda")
    kbuf[4:4 + kc.size] = dev(kc.reshape(-1))
    vbuf[4:4 + vt.size] = dev(vt.reshape(-1))
    q = (rng.standard_normal((rows, nh * hd)) * 2).astype(np.float32)
    out = torch.full((rows, nh * hd), float("nan"), device="cuda")
    D.attend_q8(out, nh * hd, dev(q), nh * hd, kbuf[4:], n * kvh * hd, dev(ks), n, vbuf[4:],
                vt.shape[1], dev(vs), n, rows, nh, kvh, hd, 0, n, 0)
    torch.cuda.synchronize()
    want = np.stack([orc.attend_q8(q[r], kc[r], ks[r], vt[r], vs[r], nh, kvh, hd, 0, n, 0)
                     for r in range(rows)])
    same(out.cpu().numpy(), want, True, "attend, 4-byte aligned caches")


def test_attention_rejects_bad_windows():
    from fastgemma_b200 import _lib
    z = torch.zeros(4096, device="cuda")
    zi = torch.zeros(4096, dtype=torch.int8, device="cuda")
    with pytest.raises(_lib.FgmCudaError, match="ring"):
        D.attend_q8(z, 256, z, 256, zi, 0, z, 0, zi, 0, z, 0, 1, 1, 1, 256, 0, 200, 128)
    with pytest.raises(_lib.FgmCudaError, match="head_dim"):
        D.attend_q8(z, 256, z, 256, zi, 0, z, 0, zi, 0, z, 0, 1, 1, 1, 96, 0, 16, 0)
    with pytest.raises(_lib.FgmCudaError, match="aligned"):
        D.attend_q8(z, 256, z, 256, zi[1:], 0, z, 0, zi, 0, z, 0, 1, 1, 1, 256, 0, 16, 0)
    with pytest.raises(_lib.FgmCudaError, match="fit"):
        D.attend_q8(z, 4096, z, 4096, zi, 0, z, 0, zi, 0, z, 0, 1, 32, 1, 64, 0, 16, 0)


def _bits_equal(got, want, what):
    got, want = np.asarray(got), np.asarray(want)
    assert got.shape == want.shape, f"{what}: shape {got.shape} vs {want.shape}"
    g = got.view(np.uint32) if got.dtype == np.float32 else got
    w = want.view(np.uint32) if want.dtype == np.float32 else want
    bad = g != w
    assert not bad.any(), f"{what}: {int(bad.sum())} of {bad.size} differ"


@pytest.mark.parametrize("rows,n,with_proj", [(5, 2048, True), (8, 2048, False), (3, 8192, True),
                                              (17, 1024, True)])
def test_norm_prep_against_oracle(orc, rows, n, with_proj):
    """Post-norm + residual add + pre-norm + prep in one launch equals the
    oracle's rmsnorm, add, rmsnorm and prep_rows: h, scales and packed rows
    bit for bit, padding rows of the last 16-row tile zeroed."""
    rng = np.random.default_rng(rows * 7 + n)
    h = rng.standard_normal((rows, n)).astype(np.float32)
    proj = (rng.standard_normal((rows, n)) * 3).astype(np.float32)
    w_post = rng.uniform(0.5, 1.5, n).astype(np.float32)
    w_pre = rng.uniform(0.5, 1.5, n).astype(np.float32)
    eps = 1e-6
    want_h = orc.add(h, orc.rmsnorm(proj, w_post, eps)) if with_proj else h
    _, _, want_qs, want_pa = orc.prep_rows(orc.rmsnorm(want_h, w_pre, eps), rows, n, 0)
    th = dev(h)
    qs = torch.empty(rows, device="cuda")
    pa = torch.full((want_pa.size,), 7, dtype=torch.int8, device="cuda")
    D.norm_prep(th, dev(proj) if with_proj else None, dev(w_post), dev(w_pre), rows, n, eps, qs, pa)
    torch.cuda.synchronize()
    _bits_equal(th.cpu().numpy(), want_h, "h")
    _bits_equal(qs.cpu().numpy(), want_qs, "scales")
    _bits_equal(pa.cpu().numpy(), want_pa, "packed rows")


@pytest.mark.parametrize("rows,n,fused", [(8, 8192, True), (3, 1024, False), (5, 192, True)])
def test_gelu_mul_prep_against_oracle(orc, rows, n, fused):
    """fused: gate and up are the two halves of one [gate | up] GEMM output."""
    rng = np.random.default_rng(rows + n)
    gate = (rng.standard_normal((rows, n)) * 2).astype(np.float32)
    up = rng.standard_normal((rows, n)).astype(np.float32)
    want_act = orc.gelu_mul(gate, up)
    _, _, want_qs, want_pa = orc.prep_rows(want_act, rows, n, 0)
    act = torch.empty((rows, n), device="cuda")
    qs = torch.empty(rows, device="cuda")
    pa = torch.full((want_pa.size,), 7, dtype=torch.int8, device="cuda")
    if fused:
        gu = dev(np.concatenate([gate, up], axis=1))
        D.gelu_mul_prep(gu, gu[:, n:], rows, n, qs, pa, act=act, ld=2 * n)
    else:
        D.gelu_mul_prep(dev(gate), dev(up), rows, n, qs, pa, act=act)
    torch.cuda.synchronize()
    _bits_equal(act.cpu().numpy(), want_act, "act")
    _bits_equal(qs.cpu().numpy(), want_qs, "scales")
    _bits_equal(pa.cpu().numpy(), want_pa, "packed rows")


@pytest.mark.parametrize("nh,kvh,hd,ring,fused", [(8, 2, 256, 0, True), (4, 1, 128, 64, False),
                                                  (8, 8, 72, 0, False)])
def test_qkv_post_equals_the_separate_kernels(orc, nh, kvh, hd, ring, fused):
    """Head norms, rope and the int8 K / V cache writes in one launch equal
    the separate glue kernels bit for bit (and the oracle's norms and rope
    to the libm tolerance)."""
    rng = np.random.default_rng(nh * hd + ring)
    rows, kvd, cap, eps = 4, kvh * hd, 160, 1e-6
    pos = np.array([5, 150, 77, 128], np.int32)
    q = (rng.standard_normal((rows, nh * hd)) * 2).astype(np.float32)
    k = (rng.standard_normal((rows, kvd)) * 2).astype(np.float32)
    v = rng.standard_normal((rows, kvd)).astype(np.float32)
    qn = rng.uniform(0.5, 1.5, hd).astype(np.float32)
    kn = rng.uniform(0.5, 1.5, hd).astype(np.float32)
    inv_freq = (1.0 / 10000.0 ** (np.arange(0, hd, 2) / hd)).astype(np.float32)
    slots = ring or cap
    vslots = (slots + 3) // 4 * 4

    def caches():
        return (torch.zeros((rows, slots, kvd), dtype=torch.int8, device="cuda"),
                torch.zeros((rows, slots), device="cuda"),
                torch.zeros((rows, vslots * kvd), dtype=torch.int8, device="cuda"),
                torch.zeros((rows, slots), device="cuda"))

    tq = dev(q)
    if fused:  # k and v: the two halves of one [k | v] GEMM output
        tkv = dev(np.concatenate([k, v], axis=1))
        tk, tv = tkv[:, :kvd], tkv[:, kvd:]
    else:
        tk, tv = dev(k), dev(v)
    kc, ks, vt, vs = caches()
    tpos, tinv = dev(pos), dev(inv_freq)
    D.qkv_post(tq, tk, tv, rows, nh, kvh, hd, dev(qn), dev(kn), eps, tinv, tpos, ring, slots,
               kc, slots * kvd, ks, slots, vt, vt.shape[1], vs, slots,
               kv_ld=2 * kvd if fused else kvd)
    # the same steps one kernel at a time
    rq, rk, rv = dev(q), dev(k), dev(v)
    D.rmsnorm(rq, rq, dev(qn), rows * nh, hd, eps)
    D.rmsnorm(rk, rk, dev(kn), rows * kvh, hd, eps)
    D.rmsnorm(rv, rv, None, rows * kvh, hd, eps)
    D.rope(rq, nh * hd, rows, nh, hd, tinv, tpos)
    D.rope(rk, kvd, rows, kvh, hd, tinv, tpos)
    k8, v8 = (torch.empty((rows, kvd), dtype=torch.int8, device="cuda") for _ in range(2))
    ksc, vsc = torch.empty(rows, device="cuda"), torch.empty(rows, device="cuda")
    D.quant_act(rk, rows, kvd, k8, ksc)
    D.quant_act(rv, rows, kvd, v8, vsc)
    rkc, rks, rvt, rvs = caches()
    for r in range(rows):
        sl = int(pos[r]) % ring if ring else int(pos[r])
        rkc[r, sl] = k8[r]
        rks[r, sl] = ksc[r]
        rvs[r, sl] = vsc[r]
        D.store_v_t(rvt[r:r + 1], rvt.shape[1], v8[r:r + 1], kvd, 1, kvd, sl)
    torch.cuda.synchronize()
    for got, want, what in ((tq, rq, "q"), (tk, rk, "k"), (tv, rv, "v"), (kc, rkc, "K cache"),
                            (ks, rks, "K scales"), (vt, rvt, "V cache"), (vs, rvs, "V scales")):
        _bits_equal(got.cpu().numpy(), want.cpu().numpy(), what)
    oq = orc.rope(orc.rmsnorm(q.reshape(-1, hd), qn, eps).reshape(rows, -1)[0], nh, hd, inv_freq,
                  int(pos[0]))
    same(tq.cpu().numpy()[0], oq, False, "q against the oracle")
    # rope's cos / sin from the host's libm table: q and k of every row equal
    # the oracle's norms and rope bit for bit where the head norm has no
    # scalar tail (head_dim % 16 == 0)
    cs = dev(D.rope_table(cap, hd, inv_freq))
    tq, tk, tv = dev(q), dev(k), dev(v)
    kc, ks, vt, vs = caches()
    D.qkv_post(tq, tk, tv, rows, nh, kvh, hd, dev(qn), dev(kn), eps, tinv, tpos, ring, slots,
               kc, slots * kvd, ks, slots, vt, vt.shape[1], vs, slots, cs=cs)
    torch.cuda.synchronize()
    for got, x, n, w, what in ((tq, q, nh, qn, "q"), (tk, k, kvh, kn, "k")):
        want = np.stack([orc.rope(orc.rmsnorm(x[r].reshape(-1, hd), w, eps).reshape(-1), n, hd,
                                  inv_freq, int(pos[r])) for r in range(rows)])
        same(got.cpu().numpy(), want, hd % 16 == 0, f"{what} with the table against the oracle")


def test_qkv_post_writes_no_cache_entry_outside_the_capacity():
    """A row whose position falls outside its cache (no ring) keeps its q / k
    / v results but writes no K / V entry; the other rows write theirs."""
    rng = np.random.default_rng(3)
    rows, nh, kvh, hd, cap = 2, 4, 1, 64, 8
    kvd = kvh * hd
    q = dev(rng.standard_normal((rows, nh * hd)).astype(np.float32))
    k = dev(rng.standard_normal((rows, kvd)).astype(np.float32))
    v = dev(rng.standard_normal((rows, kvd)).astype(np.float32))
    ones = torch.ones(hd, device="cuda")
    inv_freq = dev((1.0 / 10000.0 ** (np.arange(0, hd, 2) / hd)).astype(np.float32))
    pos = dev(np.array([3, 8], np.int32))  # row 1: slot 8 of an 8-slot cache
    kc = torch.zeros((rows, cap, kvd), dtype=torch.int8, device="cuda")
    ks = torch.zeros((rows, cap), device="cuda")
    vt = torch.zeros((rows, cap * kvd), dtype=torch.int8, device="cuda")
    vs = torch.zeros((rows, cap), device="cuda")
    D.qkv_post(q, k, v, rows, nh, kvh, hd, ones, ones, 1e-6, inv_freq, pos, 0, cap, kc, cap * kvd,
               ks, cap, vt, cap * kvd, vs, cap)
    torch.cuda.synchronize()
    assert ks[0, 3].item() > 0 and vs[0, 3].item() > 0 and kc[0, 3].abs().sum().item() > 0
    assert ks[1].abs().sum().item() == 0 and vs[1].abs().sum().item() == 0
    assert kc[1].abs().sum().item() == 0 and vt[1].abs().sum().item() == 0
    assert torch.isfinite(q).all() and k[1].abs().sum().item() > 0


def test_decode_step_matches_the_oracle_end_to_end(orc):
    """A small decode step built from the device entries the config-3 bench
    uses (norm_prep, one [q|k|v] GEMM, qkv_post, attention, prep, o GEMM,
    norm_prep, [gate|up] GEMM, gelu_mul_prep, down GEMM, norm_prep; then the
    LM head and softcap) against the same step composed from the oracle's
    restatements (pinned to the reference's own composed step in
    test_oracle.py).  Rope's cos / sin come from the host's libm table
    (fgm_cuda_rope_table, what the reference calls per position) and every
    row length and the attention window are multiples of 16 (no libm
    tails), so the logits, tokens and the cache entries written are equal
    bit for bit."""
    import decode_step
    d = decode_step.DIMS
    M, H, NH, KVH, HD, FF, T, L, V, G64, eps = (d[k] for k in
                                                "M H NH KVH HD FF T L V G eps".split())
    inp = decode_step.make_inputs()
    QKV, QD, KVD, pos, vslots = inp["QKV"], inp["QD"], inp["KVD"], inp["pos"], inp["vslots"]
    want, _, want_ks, _, _ = decode_step.compose(orc, inp)
    want_tok = orc.argmax_rows(want)

    t = lambda a: dev(a)  # noqa: E731
    dl = [{k: ((t(v[0]), t(v[1])) if isinstance(v, tuple) else t(v)) for k, v in lw.items()}
          for lw in inp["layers"]]
    tx, tinv = t(inp["x"]), t(inp["inv_freq"])
    cs = t(D.rope_table(T, HD, inp["inv_freq"]))
    tpos = torch.full((M,), pos, dtype=torch.int32, device="cuda")
    tkc, tks, tvt, tvs = t(inp["kc"]), t(inp["ks"]), t(inp["vt"]), t(inp["vs"])
    qs = torch.empty(M, device="cuda")
    pa = {k: D.packed_a(M, k, torch.device("cuda")) for k in (H, FF)}
    qkv = torch.empty((M, QKV), device="cuda")
    attn, o = torch.empty((M, QD), device="cuda"), torch.empty((M, H), device="cuda")
    gu, dn = torch.empty((M, 2 * FF), device="cuda"), torch.empty((M, H), device="cuda")
    logits = torch.empty((M, V), device="cuda")
    D.norm_prep(tx, None, None, dl[0]["inw"], M, H, eps, qs, pa[H])
    for li, lw in enumerate(dl):
        D.gemm_q4g(M, QKV, H, pa[H], qs, lw["qkv"][0], lw["qkv"][1], G64, qkv)
        D.qkv_post(qkv[:, :QD], qkv[:, QD:QD + KVD], qkv[:, QD + KVD:], M, NH, KVH, HD, lw["qn"],
                   lw["kn"], eps, tinv, tpos, 0, T, tkc[li], T * KVD, tks[li], T, tvt[li],
                   vslots * KVD, tvs[li], T, q_ld=QKV, kv_ld=QKV, cs=cs)
        D.attend_q8(attn, QD, qkv, QKV, tkc[li], T * KVD, tks[li], T, tvt[li], vslots * KVD,
                    tvs[li], T, M, NH, KVH, HD, 0, T)
        D.prep_rows(attn, QD, qs, pa[H], M, QD, 0)
        D.gemm_q4g(M, H, QD, pa[H], qs, lw["o"][0], lw["o"][1], G64, o)
        D.norm_prep(tx, o, lw["pa"], lw["pf"], M, H, eps, qs, pa[H])
        D.gemm_q4g(M, 2 * FF, H, pa[H], qs, lw["gu"][0], lw["gu"][1], G64, gu)
        D.gelu_mul_prep(gu, gu[:, FF:], M, FF, qs, pa[FF], ld=2 * FF)
        D.gemm_q4g(M, H, FF, pa[FF], qs, lw["dn"][0], lw["dn"][1], G64, dn)
        D.norm_prep(tx, dn, lw["pff"], dl[li + 1]["inw"] if li + 1 < L else t(inp["fin"]), M, H,
                    eps, qs, pa[H])
    D.gemm_q4g(M, V, H, pa[H], qs, t(inp["lm"][0]), t(inp["lm"][1]), G64, logits)
    D.softcap(logits, M, V, 30.0)
    torch.cuda.synchronize()
    got = logits.cpu().numpy()
    bad = got.view(np.uint32) != want.view(np.uint32)
    assert not bad.any(), f"{int(bad.sum())} logits differ, max |diff| {np.abs(got - want).max()}"
    assert np.array_equal(orc.argmax_rows(got), want_tok)
    got_ks = tks.cpu().numpy()
    assert np.array_equal(got_ks[:, :, :pos], inp["ks"][:, :, :pos])  # old slots untouched
    assert np.array_equal(got_ks.view(np.uint32), want_ks.view(np.uint32))
