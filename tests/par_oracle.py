"""Threaded calls of the scalar C oracle and exact NumPy checksums, for parity
checks at full BASELINE sizes.  Test infrastructure only.

The oracle's entry points take a column range [n0, n1) in n-blocks and write
only those columns, so disjoint ranges run in parallel host threads (ctypes
releases the GIL for the duration of each C call).
"""
from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np


def _ranges(n0: int, n1: int, parts: int):
    step = max(1, -(-(n1 - n0) // parts))
    return [(a, min(a + step, n1)) for a in range(n0, n1, step)]


def gemm_q8c(orc, M, N, K, pa, a_scale, b, b_scale, c, ldc, n0, n1, threads=None):
    """orc.gemm_q8c over n-blocks [n0, n1) into c [M, ldc], split over threads."""
    threads = threads or os.cpu_count() or 1
    with ThreadPoolExecutor(threads) as ex:
        list(ex.map(lambda r: orc.gemm_q8c(M, N, K, pa, a_scale, b, b_scale, c=c, ldc=ldc,
                                           n0=r[0], n1=r[1]),
                    _ranges(n0, n1, 4 * threads)))
    return c


def gemm_q4g(orc, M, N, K, pa, a_scale, bq, b_scale, group, c, ldc, n0, n1, threads=None):
    threads = threads or os.cpu_count() or 1
    with ThreadPoolExecutor(threads) as ex:
        list(ex.map(lambda r: orc.gemm_q4g(M, N, K, pa, a_scale, bq, b_scale, group, c=c,
                                           ldc=ldc, n0=r[0], n1=r[1]),
                    _ranges(n0, n1, 4 * threads)))
    return c


def q8c_rows(b: np.ndarray, N: int, K: int) -> np.ndarray:
    """The .fgm int8 tile blob [N/16][K/64][k/4 (16)][n (16)][k%4 (4)] as W [N, K]
    (convert/quant.py:96-117)."""
    t = b.reshape(N // 16, K // 64, 16, 16, 4).transpose(0, 3, 1, 2, 4)
    return np.ascontiguousarray(t).reshape(N, K)


def q8c_acc_checksums(A, b, N: int, K: int, chunk: int = 1024):
    """Exact row and column sums of acc = A @ W^T (the int32 accumulators of an
    int8 GEMM) without forming acc:  sum_n acc[m, n] = A[m] . (sum_n W[n]) and
    sum_m acc[m, n] = (sum_m A[m]) . W[n].  A: int8 [M, K] and b: the .fgm
    int8 tile blob, as torch tensors on any device (the weight is read in its
    tile order, `chunk` n-blocks at a time).  Float64 arithmetic is exact
    here, in any summation order: every partial sum is an integer below 2^53
    for int8 operands, K <= 65536 and M, N <= 2^20.  Returns
    (row_sums [M], col_sums [N]) as int64 tensors on A's device."""
    import torch
    f64 = torch.float64
    Af = A.to(f64)
    asum = Af.sum(dim=0).reshape(K // 64, 16, 4)  # k = kt*64 + j*4 + i
    wsum = torch.zeros((K // 64, 16, 4), dtype=f64, device=A.device)
    col = torch.empty(N, dtype=f64, device=A.device)
    nbs = N // 16
    for nb0 in range(0, nbs, chunk):
        nb1 = min(nbs, nb0 + chunk)
        sub = b[nb0 * 16 * K:nb1 * 16 * K].reshape(nb1 - nb0, K // 64, 16, 16, 4).to(f64)
        wsum += sub.sum(dim=(0, 3))
        col[nb0 * 16:nb1 * 16] = torch.einsum("bkjci,kji->bc", sub, asum).reshape(-1)
        del sub
    row = Af @ wsum.reshape(K)
    return row.to(torch.int64), col.to(torch.int64)
