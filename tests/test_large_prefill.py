"""Parity of the tcgen05 int8 GEMM at BASELINE's full prefill sizes.

Config 2 (M=256, K=2048, N=16384, and the K=8192, N=2048 down projection):
every output element against the scalar oracle, which runs in host threads.

Config 4 (M in {256, 1024, 4096} x K=2048 x N=262144, the LM-head width): the
scalar oracle cannot cover 2.2 T multiply-adds in a test, so the full output
is checked through exact properties instead:
  * column blocks spread over the width, including the first and the last,
    bit-exact against the oracle (f32 outputs and int32 accumulators);
  * every row sum and every column sum of the int32 accumulators equal the
    exact sums A[m].(sum_n W[n]) and (sum_m A[m]).W[n] (linearity; computed
    from the oracle's int8 activations and the weight bytes in float64, exact
    for these sizes), so an error anywhere in the accumulators shows;
  * every f32 output equals the reference epilogue applied to its
    accumulator, (float)acc * (b_scale[n] * a_scale[m])
    (amx_gemm.c:399), evaluated in torch float32 (IEEE round-to-nearest).
Reference: fgm_gemm_q8c (amx_gemm.c:444-475), fgm_gemm_q8c_vnni
(vnni_gemm.c:224-245); the LM head these shapes stand for is called at
fgm-core/src/forward.rs:687.
"""
import numpy as np
import pytest

import fastgemma_b200 as fg
import fastgemma_b200.device  # noqa: F401  (binds fg.device)
from fastgemma_b200 import fgm_format as F
import par_oracle as P

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", autouse=True)
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)


def D(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _status_ok():
    from fastgemma_b200 import _lib
    return _lib.lib().fgm_cuda_device_status() == 0


@pytest.mark.parametrize("K,N", [(2048, 16384), (8192, 2048)])
def test_config2_full_width_against_the_oracle(orc, K, N):
    """BASELINE config 2 at full size: prep of X ~ N(0,1) on the device, then
    the tensor-core GEMM; every element bit-exact against the oracle's prep
    and GEMM (threaded over column ranges)."""
    M = 256
    x = F.synth_x(M, K, 21 + K)
    b, s = F.synth_q8c(N, K, 22 + N, structured=False)
    _, qa_ref, qs_ref, pa_ref = orc.prep_rows(x, M, K, 0)
    bd, sd = D(b), D(s)
    fg.device.q8c_prepare(bd, N, K)
    try:
        xd = D(x)
        pa = fg.device.packed_a(M, K, xd.device)
        qs = torch.empty(M, device="cuda")
        qa = torch.empty((M, K), dtype=torch.int8, device="cuda")
        fg.device.prep_rows(xd, K, qs, pa, M, K, 0, qa=qa)
        c_rows = torch.full((M, N), -5.0, device="cuda")
        fg.device.gemm_q8c_rows(M, N, K, qa, qs, bd, sd, c_rows)  # the bench's prefill entry
        c_packed = torch.full((M, N), -5.0, device="cuda")
        fg.device.gemm_q8c(M, N, K, pa, qs, bd, sd, c_packed)
        torch.cuda.synchronize()
        assert _status_ok()
        assert np.array_equal(pa.cpu().numpy(), pa_ref)
        assert np.array_equal(qs.cpu().numpy().view(np.uint32), qs_ref.view(np.uint32))
        want = np.zeros((M, N), np.float32)
        P.gemm_q8c(orc, M, N, K, pa_ref, qs_ref, b, s, want, N, 0, N // 16)
        for got in (c_rows.cpu().numpy(), c_packed.cpu().numpy()):
            same = got.view(np.uint32) == want.view(np.uint32)
            assert same.all(), f"{int((~same).sum())} of {M * N} outputs differ"
    finally:
        fg.device.q8c_release(bd)


@pytest.fixture(scope="module")
def lm_head_int8():
    """The config-4 weight: int8 N=262144 x K=2048 (uniform in [-127, 127],
    drawn as tile bytes), per-channel scales U(0.001, 0.01), on host and device,
    prepared once for the tensor cores."""
    N, K = 262144, 2048
    gen = torch.Generator(device="cuda")
    gen.manual_seed(404)  # drawn on the device: 512 MiB of host RNG takes too long
    bd = torch.randint(-127, 128, (N * K,), dtype=torch.int8, device="cuda", generator=gen)
    sd = torch.empty(N, device="cuda").uniform_(0.001, 0.01, generator=gen)
    b, s = bd.cpu().numpy(), sd.cpu().numpy()
    fg.device.q8c_prepare(bd, N, K)
    yield N, K, b, s, bd, sd
    fg.device.q8c_release(bd)
    del bd, sd
    torch.cuda.empty_cache()


@pytest.mark.parametrize("M", [256, 1024, 4096])
def test_config4_lm_head_width(orc, lm_head_int8, M):
    N, K, b, s, bd, sd = lm_head_int8
    x = F.synth_x(M, K, 40 + M)
    _, qa_ref, qs_ref, pa_ref = orc.prep_rows(x, M, K, 0)
    xd = D(x)
    qs = torch.empty(M, device="cuda")
    qa = torch.empty((M, K), dtype=torch.int8, device="cuda")
    pa = fg.device.packed_a(M, K, xd.device)
    fg.device.prep_rows(xd, K, qs, pa, M, K, 0, qa=qa)
    c = torch.empty((M, N), device="cuda")
    fg.device.gemm_q8c_rows(M, N, K, qa, qs, bd, sd, c)
    acc = torch.empty((M, N), dtype=torch.int32, device="cuda")
    fg.device.gemm_q8c_acc(M, N, K, pa, bd, acc)
    torch.cuda.synchronize()
    assert _status_ok()
    assert np.array_equal(qa.cpu().numpy(), qa_ref)
    assert np.array_equal(qs.cpu().numpy().view(np.uint32), qs_ref.view(np.uint32))

    # 1. sampled column blocks, f32 and int32, against the oracle
    nbs = N // 16
    blocks = [0, 4, nbs // 3 // 4 * 4, nbs // 2, nbs - 4 * 7, nbs - 4]
    want = np.zeros((M, N), np.float32)
    for nb in blocks:
        P.gemm_q8c(orc, M, N, K, pa_ref, qs_ref, b, s, want, N, nb, nb + 4)
    for nb in blocks:
        cols = slice(nb * 16, (nb + 4) * 16)
        got = c[:, cols].cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want[:, cols].view(np.uint32)), f"nb {nb}"
        got_acc = acc[:, cols].cpu().numpy()
        want_acc = orc.gemm_q8c_acc(M, N, K, pa_ref, b, nb, nb + 4)[:, cols]
        assert np.array_equal(got_acc, want_acc), f"acc nb {nb}"

    # 2. every row and column sum of the accumulators, exact
    # (the exact expected sums come from the oracle's activations and the
    # weight bytes, in float64 torch arithmetic on the device)
    row_want, col_want = P.q8c_acc_checksums(D(qa_ref), bd, N, K)
    row_got = torch.empty(M, dtype=torch.int64, device="cuda")
    col_got = torch.zeros(N, dtype=torch.int64, device="cuda")
    for m0 in range(0, M, 256):
        blk = acc[m0:m0 + 256].to(torch.int64)
        row_got[m0:m0 + 256] = blk.sum(dim=1)
        col_got += blk.sum(dim=0)
        del blk
    assert torch.equal(row_got, row_want)
    assert torch.equal(col_got, col_want)

    # 3. every f32 output is the reference epilogue of its accumulator
    for m0 in range(0, M, 256):
        ref = acc[m0:m0 + 256].to(torch.float32) * (sd[None, :] * qs[m0:m0 + 256, None])
        assert torch.equal(ref.view(torch.int32), c[m0:m0 + 256].view(torch.int32)), \
            f"f32 epilogue differs in rows [{m0}, {m0 + 256})"
    del c, acc
    torch.cuda.empty_cache()
