"""Generate the committed golden vectors in ``tests/golden/golden.npz``.

Run in a tree where the reference is available (its ``convert/`` package and
its C kernels compiled into ``oracle/_ref`` by ``make -C oracle ref``):

    python tests/golden/make_golden.py [--ref /path/to/fastgemma]

Every expected value here comes from the reference itself:

* format pins -- ``convert/quant.py``'s ``pack_b_tiles`` / ``pack_nibbles``
  (quant.py:76-107) applied to seeded integer weights;
* GEMM outputs -- the reference kernels ``fgm_gemm_q4g`` / ``fgm_gemm_q8c``
  (AMX, amx_gemm.c:333-475) on the exact inputs of the reference's own
  harnesses (bench/kernels/vnni_test.c, gemm_test.c), after checking that the
  VNNI kernels (vnni_gemm.c:224-322) agree bit for bit;
* int32 accumulators -- the same kernels run with unit scales, where
  C == float(acc) exactly while |acc| < 2^24;
* prep -- ``fgm_prep_rows`` (ops.c:293-314) on seeded rows.

Inputs are not stored: they are rebuilt from the harness PRNGs
(``tests/golden/harness.py``); a SHA-256 of each input is stored so drift in
the rebuild is caught.  Outputs are stored as SHA-256 digests, with the full
arrays kept for the smaller cases.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, HERE)

from oracle.oracle import Oracle, Reference  # noqa: E402
import harness  # noqa: E402

FULL_LIMIT = 8192  # store full output arrays up to this many elements


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def load_quant(ref_root: str):
    spec = importlib.util.spec_from_file_location(
        "ref_quant", os.path.join(ref_root, "convert", "quant.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def pack_ref(ref, M, K, A):
    ap = np.zeros(((M + 15) // 16) * 16 * K, np.int8)
    ref.lib.fgm_pack_a(M, K, A.ctypes.data, ap.ctypes.data)
    return ap


def main():
    ap_ = argparse.ArgumentParser()
    ap_.add_argument("--ref", default=os.environ.get("FGM_REFERENCE") or os.path.join(
        os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))), "reference"))
    args = ap_.parse_args()
    orc = Oracle()
    ref = Reference()
    assert ref.has_amx and ref.has_vnni, "golden vectors need both AMX and VNNI paths"
    assert ref.backend == "amx"
    quant = load_quant(args.ref)
    out: dict[str, np.ndarray] = {}
    meta: list[str] = []

    # ---------------------------------------------------------- format pins
    rng_state = np.array([0x9E3779B97F4A7C15], np.uint64)
    for (n, k) in [(16, 64), (32, 128), (48, 256)]:
        w8 = orc.xorshift(rng_state, -127, 127, n * k).astype(np.int8).reshape(n, k)
        w4 = orc.xorshift(rng_state, -8, 7, n * k).astype(np.int8).reshape(n, k)
        tag = f"fmt_{n}x{k}"
        out[tag + "_w8_sha"] = np.array(sha(w8))
        out[tag + "_w4_sha"] = np.array(sha(w4))
        out[tag + "_tiles8"] = quant.pack_b_tiles(w8, n, k).astype(np.int8)
        out[tag + "_tiles4"] = quant.pack_nibbles(quant.pack_b_tiles(w4, n, k)).astype(np.uint8)
        meta.append(tag)
    out["fmt_state_after"] = rng_state.copy()

    # ------------------------------------------------- vnni_test.c cases
    for idx, (case, A, a_scale, B, b_scale) in enumerate(harness.vnni_test_inputs(orc)):
        kind, M, N, K, group, n0, n1 = case
        ap = pack_ref(ref, M, K, A)
        tag = f"vnni_{idx:02d}_{kind}_M{M}_N{N}_K{K}" + (f"_g{group}" if group else "")
        if kind == "q8c":
            c_amx = ref.gemm_q8c(M, N, K, ap, a_scale, B, b_scale, n0=n0, n1=n1, backend="amx")
            c_vnni = ref.gemm_q8c(M, N, K, ap, a_scale, B, b_scale, n0=n0, n1=n1, backend="vnni")
        else:
            c_amx = ref.gemm_q4g(M, N, K, ap, a_scale, B, b_scale, group, n0=n0, n1=n1,
                                 backend="amx")
            c_vnni = ref.gemm_q4g(M, N, K, ap, a_scale, B, b_scale, group, n0=n0, n1=n1,
                                  backend="vnni")
        assert np.array_equal(c_amx.view(np.uint32), c_vnni.view(np.uint32)), tag
        out[tag + "_in_sha"] = np.array(sha(A) + sha(B) + sha(a_scale) + sha(b_scale))
        out[tag + "_C_sha"] = np.array(sha(c_amx))
        if c_amx.size <= FULL_LIMIT:
            out[tag + "_C"] = c_amx
        meta.append(tag)

    # ------------------------------------------------- gemm_test.c case
    g = harness.gemm_test_inputs(orc)
    M, N, K, group = g["M"], g["N"], g["K"], g["group"]
    ap = pack_ref(ref, M, K, g["A"])
    ap8 = pack_ref(ref, 8, K, g["A"][:8])
    c4 = ref.gemm_q4g(M, N, K, ap, g["a_scale"], g["Bq"], g["bs4"], group, backend="amx")
    c8 = ref.gemm_q8c(M, N, K, ap, g["a_scale"], g["B8"], g["bs8"], backend="amx")
    c4d = ref.gemm_q4g(8, N, K, ap8, g["a_scale"], g["Bq"], g["bs4"], group, backend="amx")
    assert np.array_equal(c4, ref.gemm_q4g(M, N, K, ap, g["a_scale"], g["Bq"], g["bs4"], group,
                                           backend="vnni"))
    out["gemmtest_in_sha"] = np.array(sha(g["A"]) + sha(g["Bq"]) + sha(g["B8"]) +
                                      sha(g["bs4"]) + sha(g["bs8"]) + sha(g["a_scale"]))
    out["gemmtest_q4g_C"] = c4
    out["gemmtest_q8c_C"] = c8
    out["gemmtest_q4g_decode_C"] = c4d[:8]
    meta.append("gemmtest")

    # --------------------------------------- int32 accumulators (unit scales)
    st = np.array([0x51ED2701], np.uint64)
    for (kind, M, N, K) in [("q8c", 16, 128, 2048), ("q8c", 8, 64, 8192),
                            ("q4g", 16, 128, 2048), ("q4g", 5, 64, 8192)]:
        A = orc.xorshift(st, -127, 127, M * K).astype(np.int8).reshape(M, K)
        ap = pack_ref(ref, M, K, A)
        ones_a = np.ones(M, np.float32)
        tag = f"acc_{kind}_M{M}_N{N}_K{K}"
        if kind == "q8c":
            B = orc.xorshift(st, -127, 127, N * K).astype(np.int8)
            c = ref.gemm_q8c(M, N, K, ap, ones_a, B, np.ones(N, np.float32), backend="amx")
        else:
            B = orc.xorshift(st, 0, 255, N * K // 2).astype(np.uint8)
            c = ref.gemm_q4g(M, N, K, ap, ones_a, B, np.ones((1, N), np.float16), K,
                             backend="amx")
        assert np.all(np.abs(c) < 2.0 ** 24), tag  # exact float(acc)
        assert np.array_equal(c, np.round(c))
        out[tag + "_in_sha"] = np.array(sha(A) + sha(B))
        out[tag + "_acc"] = c.astype(np.int32)
        meta.append(tag)

    # ------------------------------------------------------------------ prep
    prep_cases = [(1, 2048, 2048, 0), (8, 2048, 2048, 128), (17, 2048, 2176, 128),
                  (5, 512, 512, 8), (3, 256, 256, 16), (16, 8192, 8192, 128),
                  (2, 1024, 1024, 1024), (33, 512, 520, 64)]
    for idx, (m, k, lda, hsz) in enumerate(prep_cases):
        x = harness.prep_input(orc, m, lda, seed=1000 + idx)
        if idx == 1:
            x[3, :] = 0.0  # all-zero row: scale 1.0
        if idx == 0:
            x[0, :] = 0.0  # ties: amax 127 -> s = 1 -> x*inv exact halves
            x[0, :8] = [127.0, 2.5, 3.5, -2.5, -3.5, 0.5, -0.5, 126.5]
        rot, qa, qs, pa = ref.prep_rows(x[:, :k] if lda == k else x.reshape(-1), m, k, hsz,
                                        lda=lda)
        tag = f"prep_{idx}_m{m}_k{k}_lda{lda}_h{hsz}"
        out[tag + "_in_sha"] = np.array(sha(x))
        out[tag + "_qs"] = qs
        out[tag + "_rot_sha"] = np.array(sha(rot))
        out[tag + "_qa_sha"] = np.array(sha(qa))
        out[tag + "_pa_sha"] = np.array(sha(pa))
        if qa.size <= FULL_LIMIT:
            out[tag + "_qa"] = qa
        meta.append(tag)

    out["cases"] = np.array(meta)
    path = os.path.join(HERE, "golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {len(meta)} cases, {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    main()
