"""Column-sharded LM head over NCCL, one process per GPU (needs >= 2 GPUs;
skipped otherwise).  Every rank's gathered logits must equal the oracle's
whole GEMM bit for bit."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _rank_main(rank, world, port, out_dir, fused=False):
    import torch.distributed as dist
    from datetime import timedelta
    import fastgemma_b200.device as D
    from fastgemma_b200 import fgm_format as F
    from fastgemma_b200 import shard as S
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    try:
        M, N, K = 8, 16384, 2048
        blob, scale = F.synth_q4g(N, K, 64, 33, structured=False)
        rng = np.random.default_rng(5)
        x = rng.standard_normal((M, K)).astype(np.float32)
        xd = torch.from_numpy(x).to(dev)
        pa = D.packed_a(M, K, dev)
        qs = torch.empty(M, device=dev)
        D.prep_rows(xd, K, qs, pa, M, K, 128)  # every rank quantises the same X
        sh = S.ColumnShardedGemm("q4g", blob, scale, N, K, 64, device=dev, fused=fused)
        for call in range(3 if fused else 1):  # the fused path alternates its double buffers
            out = sh(M, pa, qs)
            torch.cuda.synchronize()
            np.save(os.path.join(out_dir, f"r{rank}_c{call}.npy"), out.cpu().numpy())
        tok = sh.argmax(M, pa, qs)  # NCCL path: pairs exchanged; fused path: gathered logits scanned
        torch.cuda.synchronize()
        np.save(os.path.join(out_dir, f"r{rank}_tok.npy"), tok.cpu().numpy())
        sh.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fused", [False, True])
def test_column_sharded_lm_head(orc, tmp_path, fused):
    """fused=False: local GEMM + NCCL all-gather; fused=True: one kernel per
    rank storing its columns into every peer's output over NVLink."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two or more GPUs")
    from fastgemma_b200 import fgm_format as F
    world = min(torch.cuda.device_count(), 8)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.start_processes(_rank_main, args=(world, port, str(tmp_path), fused), nprocs=world,
                       join=True, start_method="spawn")
    M, N, K = 8, 16384, 2048
    blob, scale = F.synth_q4g(N, K, 64, 33, structured=False)
    x = np.random.default_rng(5).standard_normal((M, K)).astype(np.float32)
    _, _, qs, pa = orc.prep_rows(x, M, K, 128)
    want = orc.gemm_q4g(M, N, K, pa, qs, blob, scale, 64)
    for r in range(world):
        tok = np.load(os.path.join(tmp_path, f"r{r}_tok.npy"))
        assert np.array_equal(tok, orc.argmax_rows(want)), f"rank {r} argmax"
        for call in range(3 if fused else 1):
            got = np.load(os.path.join(tmp_path, f"r{r}_c{call}.npy"))
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"rank {r} call {call}"
