"""fgm_cuda_gemm_q8c_noalloc: the tensor-core int8 GEMM with its activation
copy in the library's fixed device buffer instead of temporary memory.

For callers that cannot allocate device memory while serving: an engine whose
HBM budget is fully reserved for weights and the KV cache at start-up, or a
host language that reaches this library only through the C ABI and has no say
over the process's CUDA memory pools.

Each case makes two calls in a row on one stream and checks both outputs
bit-exactly against the scalar oracle (orc.gemm_q8c, the reference's
arithmetic) and against the allocating entry fgm_cuda_gemm_q8c; the columns
outside [n0, n1) must stay untouched.  After a first (set-up) call, the two
calls must take nothing from the device's stream-ordered memory pool and
must not lower the device's free memory.  The file is collected last, so a
run that stops at the first failure has run every other test before it.
"""
import ctypes

import numpy as np
import pytest

import fastgemma_b200 as fg
import fastgemma_b200.device  # noqa: F401  (binds fg.device)
from fastgemma_b200 import _lib
from fastgemma_b200 import fgm_format as F

REL_TOL = 1e-5  # the f32 bound north_star states; the outputs are in fact bit-exact
STATIC_ROWS_BYTES = 4 << 20
CU_MEMPOOL_ATTR_USED_MEM_HIGH = 8


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


class _DriverMemory:
    """The device's default stream-ordered pool and free memory, through the
    CUDA driver API (the pool is shared by every runtime in the process)."""

    def __init__(self, ordinal: int):
        self.cu = ctypes.CDLL("libcuda.so.1")
        dev = ctypes.c_int()
        assert self.cu.cuDeviceGet(ctypes.byref(dev), ordinal) == 0
        self.pool = ctypes.c_void_p()
        assert self.cu.cuDeviceGetDefaultMemPool(ctypes.byref(self.pool), dev) == 0

    def reset_high(self):
        zero = ctypes.c_uint64(0)
        assert self.cu.cuMemPoolSetAttribute(self.pool, CU_MEMPOOL_ATTR_USED_MEM_HIGH,
                                             ctypes.byref(zero)) == 0

    def used_high(self) -> int:
        v = ctypes.c_uint64()
        assert self.cu.cuMemPoolGetAttribute(self.pool, CU_MEMPOOL_ATTR_USED_MEM_HIGH,
                                             ctypes.byref(v)) == 0
        return v.value

    def free_bytes(self) -> int:
        free, total = ctypes.c_size_t(), ctypes.c_size_t()
        assert self.cu.cuMemGetInfo_v2(ctypes.byref(free), ctypes.byref(total)) == 0
        return free.value


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,N,n0,n1", [(1, 2048, 256, 0, 16), (8, 1024, 128, 4, 8),
                                         (63, 2048, 192, 0, 12), (100, 1024, 384, 4, 20),
                                         (256, 2048, 512, 0, 32), (256, 16384, 128, 0, 8)])
def test_noalloc_matches_the_oracle_two_calls_in_a_row(orc, M, K, N, n0, n1):
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
            pa = F.pack_a(A)
            ins.append((pa, a_s, torch.from_numpy(pa).cuda(), torch.from_numpy(a_s).cuda()))
        ldc = N + 16
        got = [torch.full((M, ldc), -3.0, device="cuda") for _ in ins]
        alloc = [torch.full((M, ldc), -3.0, device="cuda") for _ in ins]
        warm = torch.full((M, ldc), -3.0, device="cuda")
        for (_, _, pa_d, as_d), c in zip(ins, alloc):  # the allocating entry first
            fg.device.gemm_q8c(M, N, K, pa_d, as_d, bd, sd, c, ldc, n0, n1)
        # set-up call: resolves the static buffer's address on this device
        fg.device.gemm_q8c_noalloc(M, N, K, ins[0][2], ins[0][3], bd, sd, warm, ldc, n0, n1)
        torch.cuda.synchronize()
        mem = _DriverMemory(torch.cuda.current_device())
        mem.reset_high()
        free0 = mem.free_bytes()
        for (_, _, pa_d, as_d), c in zip(ins, got):  # back to back on one stream
            fg.device.gemm_q8c_noalloc(M, N, K, pa_d, as_d, bd, sd, c, ldc, n0, n1)
        torch.cuda.synchronize()
        assert mem.used_high() == 0, "the no-allocation entry took memory from the CUDA pool"
        # (a pool trim after the synchronisation could only raise it)
        assert mem.free_bytes() >= free0, "device free memory dropped across the calls"
        assert _lib.lib().fgm_cuda_device_status() == 0
        untouched = np.ones(ldc, bool)
        untouched[n0 * 16:n1 * 16] = False
        for (pa, a_s, _, _), g, w in zip(ins, got, alloc):
            g, w = g.cpu().numpy(), w.cpu().numpy()
            want = orc.gemm_q8c(M, N, K, pa, a_s, b, s, ldc=ldc, n0=n0, n1=n1)
            cols = slice(n0 * 16, n1 * 16)
            assert np.all(g[:, untouched] == -3.0)
            assert np.array_equal(g[:, cols].view(np.uint32), want[:M, cols].view(np.uint32)), \
                f"max |d| vs oracle = {np.abs(g[:, cols] - want[:M, cols]).max()}"
            assert np.array_equal(g.view(np.uint32), w.view(np.uint32))
            denom = np.maximum(np.abs(want[:M, cols]), 1e-30)
            assert float(np.max(np.abs(g[:, cols] - want[:M, cols]) / denom)) <= REL_TOL
    finally:
        fg.device.q8c_release(bd)
