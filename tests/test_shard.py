"""Column sharding of large-N GEMMs (LM head): split, weight slices, and the
gathered result of world-size-2 gloo ranks against the whole GEMM."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from fastgemma_b200 import fgm_format as F
from fastgemma_b200 import shard as S


@pytest.mark.parametrize("nblocks,world", [(16384, 1), (16384, 2), (16384, 8), (1024, 3),
                                           (64, 8), (4, 2)])
def test_shard_ranges_cover_in_groups_of_four(nblocks, world):
    r = S.shard_ranges(nblocks, world)
    assert r[0][0] == 0 and r[-1][1] == nblocks
    for (a, b), (c, _) in zip(r, r[1:]):
        assert b == c
    sizes = [b - a for a, b in r]
    assert all(a % 4 == 0 and b % 4 == 0 for a, b in r)
    assert max(sizes) - min(sizes) <= 4


def test_shard_ranges_reject_partial_groups():
    with pytest.raises(ValueError):
        S.shard_nblocks(18, 2, 0)


def test_shard_slices_are_the_packed_columns():
    """A column shard of the blob is the .fgm packing of those columns."""
    N, K, group = 256, 512, 128
    rng = np.random.default_rng(1)
    q = rng.integers(-8, 8, size=(N, K), dtype=np.int8)
    s = rng.uniform(0.005, 0.02, size=(K // group, N)).astype(np.float16)
    bq = F.pack_q4g(q)
    for nb0, nb1 in S.shard_ranges(N // 16, 3):
        w, sc = F.q4g_column_shard(bq, s, N, K, nb0, nb1)
        assert np.array_equal(w, F.pack_q4g(q[nb0 * 16:nb1 * 16]))
        assert np.array_equal(sc, s[:, nb0 * 16:nb1 * 16])
    b8 = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    s8 = rng.uniform(0.001, 0.01, size=N).astype(np.float32)
    for nb0, nb1 in S.shard_ranges(N // 16, 2):
        w, sc = F.q8c_column_shard(F.pack_b_tiles(b8), s8, N, K, nb0, nb1)
        assert np.array_equal(w, F.pack_b_tiles(b8[nb0 * 16:nb1 * 16]))


def _oracle_gemm(sh, M, A, a_scale, C):
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                    "oracle"))
    from oracle import Oracle
    orc = Oracle()
    c = np.zeros((M, sh.max_cols), np.float32)
    if sh.kind == "q4g":
        orc.gemm_q4g(M, sh.cols, sh.K, A, a_scale, sh.w.numpy(), sh.s.numpy().view(np.float16),
                     sh.group, c=c, ldc=sh.max_cols)
    else:
        orc.gemm_q8c(M, sh.cols, sh.K, A, a_scale, sh.w.numpy(), sh.s.numpy(), c=c,
                     ldc=sh.max_cols)
    C.copy_(torch.from_numpy(c))


def _rank_main(rank, world, port, case, result_dir):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        kind, M, N, K = case
        if kind == "q4g":
            blob, scale = F.synth_q4g(N, K, 64, 7)
        else:
            blob, scale = F.synth_q8c(N, K, 7)
        rng = np.random.default_rng(3)
        A = F.pack_a(rng.integers(-128, 128, size=(M, K), dtype=np.int8))
        a_s = rng.uniform(0.01, 0.1, size=M).astype(np.float32)
        sh = S.ColumnShardedGemm(kind, blob, scale, N, K, 64, gemm=_oracle_gemm)
        out = sh(M, A, a_s)
        np.save(os.path.join(result_dir, f"r{rank}.npy"), out.numpy())
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("case", [("q4g", 8, 1024, 256), ("q8c", 3, 768, 128)])
def test_gloo_two_ranks_gather_the_whole_gemm(orc, tmp_path, case):
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), case, str(tmp_path)),
                       nprocs=world, join=True, start_method="spawn")
    kind, M, N, K = case
    if kind == "q4g":
        blob, scale = F.synth_q4g(N, K, 64, 7)
    else:
        blob, scale = F.synth_q8c(N, K, 7)
    rng = np.random.default_rng(3)
    A = F.pack_a(rng.integers(-128, 128, size=(M, K), dtype=np.int8))
    a_s = rng.uniform(0.01, 0.1, size=M).astype(np.float32)
    want = (orc.gemm_q4g(M, N, K, A, a_s, blob, scale, 64) if kind == "q4g"
            else orc.gemm_q8c(M, N, K, A, a_s, blob, scale))
    for r in range(world):
        got = np.load(os.path.join(tmp_path, f"r{r}.npy"))
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"rank {r}"
