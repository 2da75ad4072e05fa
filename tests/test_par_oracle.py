"""CPU checks of the full-size parity helpers (tests/par_oracle.py) against the
scalar oracle: the threaded calls write the same bits as one call, the tile
unpacking inverts the .fgm int8 layout, and the accumulator checksums equal
the sums of the oracle's own accumulators."""
import numpy as np

from fastgemma_b200 import fgm_format as F
import par_oracle as P


def test_threaded_oracle_equals_one_call(orc):
    M, N, K = 24, 320, 256
    rng = np.random.default_rng(3)
    A = rng.integers(-128, 128, size=(M, K), dtype=np.int8)
    pa = F.pack_a(A)
    a_s = rng.uniform(0.001, 0.05, size=M).astype(np.float32)
    b, s = F.synth_q8c(N, K, 5)
    one = orc.gemm_q8c(M, N, K, pa, a_s, b, s)
    many = P.gemm_q8c(orc, M, N, K, pa, a_s, b, s, np.zeros((M, N), np.float32), N, 0, N // 16,
                      threads=4)
    assert np.array_equal(one.view(np.uint32), many.view(np.uint32))
    bq, s4 = F.synth_q4g(N, K, 64, 6)
    one = orc.gemm_q4g(M, N, K, pa, a_s, bq, s4, 64)
    many = P.gemm_q4g(orc, M, N, K, pa, a_s, bq, s4, 64, np.zeros((M, N), np.float32), N, 0,
                      N // 16, threads=3)
    assert np.array_equal(one.view(np.uint32), many.view(np.uint32))


def test_tile_unpack_and_checksums(orc):
    M, N, K = 40, 192, 320
    rng = np.random.default_rng(4)
    W = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    b = F.pack_b_tiles(W)
    assert np.array_equal(P.q8c_rows(b, N, K), W)
    A = rng.integers(-128, 128, size=(M, K), dtype=np.int8)
    acc = orc.gemm_q8c_acc(M, N, K, F.pack_a(A), b)
    import torch
    row, col = P.q8c_acc_checksums(torch.from_numpy(A), torch.from_numpy(b), N, K, chunk=5)
    assert np.array_equal(row.numpy(), acc.astype(np.int64).sum(axis=1))
    assert np.array_equal(col.numpy(), acc.astype(np.int64).sum(axis=0))
