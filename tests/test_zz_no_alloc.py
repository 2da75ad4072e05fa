"""fgm_cuda_gemm_q8c_noalloc: the tensor-core int8 GEMM with its activation
copy in the library's fixed device buffer instead of temporary memory.

Checked against fgm_cuda_gemm_q8c (same prepared weight, same inputs) within
the parity tolerance, over two calls in a row; collected last so it also runs
after every other test in one session.
"""
import ctypes

import numpy as np
import pytest

import fastgemma_b200 as fg
import fastgemma_b200.device  # noqa: F401  (binds fg.device)
from fastgemma_b200 import _lib
from fastgemma_b200 import fgm_format as F

REL_TOL = 1e-5  # f32 outputs vs the reference path
STATIC_ROWS_BYTES = 4 << 20


def test_noalloc_rejects_oversize_before_touching_a_device():
    L = _lib.lib()
    K = 16384
    M = STATIC_ROWS_BYTES // K + 1
    p = ctypes.c_void_p(16)  # never dereferenced: the size check comes first
    rc = L.fgm_cuda_gemm_q8c_noalloc(M, 64, K, p, p, p, p, p, 64, 0, 4, None)
    assert rc == -1
    assert b"static activation buffer" in L.fgm_cuda_last_error()
    # exactly at the limit the size check passes (the null pointer is what fails)
    rc = L.fgm_cuda_gemm_q8c_noalloc(STATIC_ROWS_BYTES // K, 64, K, None, p, p, p, p, 64, 0, 4,
                                     None)
    assert rc == -1 and b"null pointer" in L.fgm_cuda_last_error()


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,N,n0,n1", [(256, 2048, 512, 0, 32), (100, 1024, 384, 4, 20),
                                         (256, 16384, 128, 0, 8)])
def test_noalloc_matches_gemm_q8c_two_calls_in_a_row(M, K, N, n0, n1):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)
    rng = np.random.default_rng(M + K + N)
    b, s = F.synth_q8c(N, K, 11 * N + M)
    bd = torch.from_numpy(b).cuda()
    sd = torch.from_numpy(s).cuda()
    fg.device.q8c_prepare(bd, N, K)
    try:
        ins = []
        for _ in range(2):
            A = rng.integers(-128, 128, size=(M, K), dtype=np.int8)
            a_s = rng.uniform(0.001, 0.05, size=M).astype(np.float32)
            ins.append((torch.from_numpy(F.pack_a(A)).cuda(), torch.from_numpy(a_s).cuda()))
        ldc = N + 16
        got = [torch.full((M, ldc), -3.0, device="cuda") for _ in ins]
        want = [torch.full((M, ldc), -3.0, device="cuda") for _ in ins]
        for (pa, a_s), c in zip(ins, got):  # back to back on one stream
            fg.device.gemm_q8c_noalloc(M, N, K, pa, a_s, bd, sd, c, ldc, n0, n1)
        for (pa, a_s), c in zip(ins, want):
            fg.device.gemm_q8c(M, N, K, pa, a_s, bd, sd, c, ldc, n0, n1)
        torch.cuda.synchronize()
        assert _lib.lib().fgm_cuda_device_status() == 0
        for g, w in zip(got, want):
            g, w = g.cpu().numpy(), w.cpu().numpy()
            assert g.shape == w.shape
            untouched = np.ones(ldc, bool)
            untouched[n0 * 16:n1 * 16] = False
            assert np.all(g[:, untouched] == -3.0)
            denom = np.maximum(np.abs(w), 1e-30)
            assert float(np.max(np.abs(g - w) / denom)) <= REL_TOL
    finally:
        fg.device.q8c_release(bd)
