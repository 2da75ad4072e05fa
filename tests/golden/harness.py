"""Rebuilds the inputs of the reference's own GEMM test harnesses.

``bench/kernels/vnni_test.c`` and ``bench/kernels/gemm_test.c`` draw their
operands from small PRNGs (restated in ``oracle/fgm_oracle.c``) in a fixed
order.  The functions here replay that order so that the parity suite runs the
very cases those harnesses run, and so that committed golden outputs can be
checked against inputs rebuilt on any machine.
"""
from __future__ import annotations

import numpy as np

# vnni_test.c:271-284, in call order (the PRNG state carries across cases)
VNNI_TEST_CASES = [
    ("q8c", 1, 256, 1536, None, 0, 16),
    ("q8c", 8, 256, 1536, None, 0, 16),
    ("q8c", 15, 256, 1536, None, 0, 16),
    ("q8c", 16, 256, 1536, None, 0, 16),
    ("q8c", 17, 256, 1536, None, 0, 16),
    ("q8c", 33, 512, 1536, None, 4, 12),
    ("q8c", 64, 256, 2048, None, 0, 16),
    ("q4g", 1, 256, 1536, 128, 0, 16),
    ("q4g", 8, 256, 1536, 128, 0, 16),
    ("q4g", 15, 256, 1536, 64, 0, 16),
    ("q4g", 16, 256, 1536, 256, 0, 16),
    ("q4g", 17, 256, 1536, 128, 0, 16),
    ("q4g", 33, 512, 1536, 128, 4, 12),
    ("q4g", 64, 256, 2048, 128, 0, 16),
]
VNNI_TEST_SEED = 0x243F6A8885A308D3
GEMM_TEST_SEED = 12345


def _f32(x):
    return np.float32(x)


def vnni_test_inputs(orc):
    """Yield (case, A, a_scale, B, b_scale) for every vnni_test.c case.

    vnni_test.c:131-169: A = rnd(-127,127) per element; q8c B = rnd(-127,127);
    q4g B bytes = rnd(0,255); a_scale = 0.01 + 0.001*(i%7);
    q8c b_scale = 0.02 + 0.0005*(i%11); q4g b_scale = f16(0.002 + 0.0001*(i%13)).
    """
    st = np.array([VNNI_TEST_SEED], np.uint64)
    for case in VNNI_TEST_CASES:
        kind, M, N, K, group, n0, n1 = case
        KB, NB = K // 64, N // 16
        A = orc.xorshift(st, -127, 127, M * K).astype(np.int8).reshape(M, K)
        i = np.arange(max(M, 1), dtype=np.int32)[:M]
        a_scale = (_f32(0.01) + _f32(0.001) * (i % 7).astype(np.float32)).astype(np.float32)
        if kind == "q8c":
            B = orc.xorshift(st, -127, 127, NB * KB * 1024).astype(np.int8)
            j = np.arange(N, dtype=np.int32)
            b_scale = (_f32(0.02) + _f32(0.0005) * (j % 11).astype(np.float32)).astype(np.float32)
        else:
            B = orc.xorshift(st, 0, 255, NB * KB * 512).astype(np.uint8)
            j = np.arange((K // group) * N, dtype=np.int32)
            b_scale = (_f32(0.002) + _f32(0.0001) * (j % 13).astype(np.float32)).astype(np.float16)
        yield case, A, a_scale, B, b_scale


def gemm_test_inputs(orc):
    """gemm_test.c:84-105: the M=40, N=64, K=256, group-64 case.

    Returns dict with A [40,256], a_scale, Bq (int4 blob), B8 (int8 blob),
    bs4 (f16 [4, 64]), bs8 (f32 [64]).
    """
    M, N, K, group = 40, 64, 256, 64
    KB, NB = K // 64, N // 16
    st = np.array([GEMM_TEST_SEED], np.uint32)
    A = orc.lcg(st, -127, 127, M * K).astype(np.int8).reshape(M, K)
    i = np.arange(M, dtype=np.int32)
    a_scale = (_f32(0.002) + _f32(0.001) * (i % 7).astype(np.float32)).astype(np.float32)
    # Bq[i] = (rnd(-8,7) & 0xF) | (rnd(-8,7) & 0xF) << 4, lo drawn first
    nib = orc.lcg(st, -8, 7, 2 * NB * KB * 512).reshape(-1, 2)
    Bq = ((nib[:, 0] & 0xF) | ((nib[:, 1] & 0xF) << 4)).astype(np.uint8)
    B8 = orc.lcg(st, -127, 127, NB * KB * 1024).astype(np.int8)
    j = np.arange((K // group) * N, dtype=np.int32)
    bs4 = (_f32(0.01) + _f32(0.001) * (j % 5).astype(np.float32)).astype(np.float16)
    j = np.arange(N, dtype=np.int32)
    bs8 = (_f32(0.003) + _f32(0.0005) * (j % 11).astype(np.float32)).astype(np.float32)
    return dict(M=M, N=N, K=K, group=group, A=A, a_scale=a_scale, Bq=Bq, B8=B8,
                bs4=bs4.reshape(K // group, N), bs8=bs8)


def prep_input(orc, m: int, lda: int, seed: int, outliers: bool = True) -> np.ndarray:
    """Seeded activation rows as exact binary fractions (no libm involved):
    x = rnd(-2^20, 2^20) / 2^18, with a few large outliers per row."""
    st = np.array([seed], np.uint64)
    x = orc.xorshift(st, -(1 << 20), 1 << 20, m * lda).astype(np.float32) / np.float32(1 << 18)
    x = x.reshape(m, lda)
    if outliers and lda >= 64:
        pos = orc.xorshift(st, 0, lda - 1, 2 * m).reshape(m, 2)
        for r in range(m):
            x[r, pos[r, 0]] = np.float32(37.25)
            x[r, pos[r, 1]] = np.float32(-52.5)
    return np.ascontiguousarray(x)
