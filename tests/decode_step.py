"""A small decode step with BASELINE config 3's structure at toy sizes,
composed from per-op implementations -- the oracle's restatements or the
reference's own kernels compiled from source, which expose the same methods
-- and the seeded inputs it runs on.  Used by the CPU test that pins the
composed oracle step to the reference and by the GPU test that checks the
device step against it."""
import numpy as np

DIMS = dict(M=3, H=256, NH=4, KVH=2, HD=64, FF=512, T=48, L=2, V=1024, G=64, eps=1e-6)


def make_inputs(seed=11):
    d = DIMS
    rng = np.random.default_rng(seed)
    M, H, NH, KVH, HD, FF, T, L, V, G = (d[k] for k in "M H NH KVH HD FF T L V G".split())
    KVD, QD = KVH * HD, NH * HD
    QKV = QD + 2 * KVD

    def q4(k, n):
        return (rng.integers(0, 256, n * k // 2).astype(np.uint8),
                rng.uniform(0.005, 0.02, (k // G, n)).astype(np.float16))

    def nw(n):
        return rng.uniform(0.5, 1.5, n).astype(np.float32)

    layers = [dict(qkv=q4(H, QKV), o=q4(QD, H), gu=q4(H, 2 * FF), dn=q4(FF, H), inw=nw(H),
                   qn=nw(HD), kn=nw(HD), pa=nw(H), pf=nw(H), pff=nw(H)) for _ in range(L)]
    vslots = (T + 3) // 4 * 4
    return dict(layers=layers, lm=q4(H, V), fin=nw(H),
                inv_freq=(1.0 / 10000.0 ** (np.arange(0, HD, 2) / HD)).astype(np.float32),
                kc=rng.integers(-127, 128, (L, M, T, KVD)).astype(np.int8),
                ks=rng.uniform(0.001, 0.02, (L, M, T)).astype(np.float32),
                vt=rng.integers(-127, 128, (L, M, vslots * KVD)).astype(np.int8),
                vs=rng.uniform(0.001, 0.02, (L, M, T)).astype(np.float32),
                x=rng.standard_normal((M, H)).astype(np.float32), pos=T - 1, vslots=vslots,
                QKV=QKV, QD=QD, KVD=KVD)


def compose(lib, inp):
    """forward.rs:469-654 per layer (norm, q|k|v projection, head norms, rope,
    int8 K / V into the caches, attention, o projection, post-norm and
    residual, pre-norm, gate|up projection, gelu_mul, down projection,
    post-norm and residual), then the final norm, LM head and softcap 30.
    Returns the logits and the caches after the step."""
    d = DIMS
    M, H, NH, KVH, HD, FF, T, L, V, G, eps = (d[k] for k in
                                              "M H NH KVH HD FF T L V G eps".split())
    QKV, QD, KVD, pos = inp["QKV"], inp["QD"], inp["KVD"], inp["pos"]
    inv_freq, slot = inp["inv_freq"], pos

    def linear(x, w, n, k):
        _, _, qs, pa = lib.prep_rows(x, M, k, 0)
        return lib.gemm_q4g(M, n, k, pa, qs, w[0], w[1], G)[:M]

    x = inp["x"].copy()
    kc, ks, vt, vs = (inp[k].copy() for k in ("kc", "ks", "vt", "vs"))
    for li, lw in enumerate(inp["layers"]):
        qkv = linear(lib.rmsnorm(x, lw["inw"], eps), lw["qkv"], QKV, H)
        attn = np.zeros((M, QD), np.float32)
        for r in range(M):
            qr = lib.rope(lib.rmsnorm(qkv[r, :QD].reshape(NH, HD), lw["qn"], eps).reshape(-1), NH,
                          HD, inv_freq, pos)
            kr = lib.rope(lib.rmsnorm(qkv[r, QD:QD + KVD].reshape(KVH, HD), lw["kn"], eps)
                          .reshape(-1), KVH, HD, inv_freq, pos)
            vr = lib.rmsnorm(qkv[r, QD + KVD:].reshape(KVH, HD), None, eps).reshape(-1)
            kq, ksc = lib.quant_act(kr[None])
            vq, vsc = lib.quant_act(vr[None])
            kc[li, r, slot], ks[li, r, slot], vs[li, r, slot] = kq[0], ksc[0], vsc[0]
            lib.store_v_t(vt[li, r], vq[0], slot)
            attn[r] = lib.attend_q8(qr, kc[li, r], ks[li, r], vt[li, r], vs[li, r], NH, KVH, HD, 0,
                                    T)
        x = lib.add(x, lib.rmsnorm(linear(attn, lw["o"], H, QD), lw["pa"], eps))
        gu = linear(lib.rmsnorm(x, lw["pf"], eps), lw["gu"], 2 * FF, H)
        act = lib.gelu_mul(gu[:, :FF], gu[:, FF:])
        x = lib.add(x, lib.rmsnorm(linear(act, lw["dn"], H, FF), lw["pff"], eps))
    logits = lib.softcap(linear(lib.rmsnorm(x, inp["fin"], eps), inp["lm"], V, H), 30.0)
    return logits, kc, ks, vt, vs
