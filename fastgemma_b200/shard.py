"""Large-N GEMMs split by output columns across the GPUs of one node.

The LM head (N = vocabulary, fgm-core/src/forward.rs:301, :687) and the wide
prefill products are large enough that their weight stream dominates a step
(the int4 LM head is 268 MB at K = 2048, the int8 one 537 MB).  Output
columns are independent, so rank r of G multiplies only n-blocks
[nb0_r, nb1_r) -- split in units of 4 n-blocks exactly like the reference's
thread pool splits one GEMM across threads (fgm-core/src/pool.rs:110-124) --
from its own slice of the weight: a contiguous byte range of the .fgm blob in
its [N/16][K/64] tile order (the q4g scales [K/group][N] need one strided
slice per group row).  Activations are replicated: every rank quantises the
same X.  The full output is assembled with one all-gather of the per-rank
column blocks over the process group (NCCL over NVLink on GPUs, gloo on CPU).

One process per GPU; ``torch.distributed`` is the plumbing, the GEMM is the
library's kernel on each rank's shard.
"""
from __future__ import annotations

from typing import Callable

import numpy as np
import torch
import torch.distributed as dist

from . import fgm_format as F


def split_units(total: int, nt: int, tid: int) -> tuple[int, int]:
    """Even split of ``total`` items over ``nt`` workers (pool.rs:110-116)."""
    per, extra = divmod(total, nt)
    start = tid * per + min(tid, extra)
    return start, start + per + (1 if tid < extra else 0)


def shard_nblocks(nblocks: int, world: int, rank: int) -> tuple[int, int]:
    """n-block range of ``rank``: whole groups of 4 n-blocks (pool.rs:119-124).

    Requires ``nblocks % 4 == 0`` (N % 64 == 0): the reference's pool split
    covers only whole groups of 4, and so does this one.
    """
    if nblocks % 4:
        raise ValueError(f"column sharding needs N % 64 == 0 (n-blocks={nblocks})")
    a, b = split_units(nblocks // 4, world, rank)
    return a * 4, b * 4


def shard_ranges(nblocks: int, world: int) -> list[tuple[int, int]]:
    return [shard_nblocks(nblocks, world, r) for r in range(world)]


def assemble(gathered: torch.Tensor, ranges: list[tuple[int, int]], out: torch.Tensor) -> torch.Tensor:
    """Place rank g's column block ``gathered[g, :, :cols_g]`` at columns
    ``[nb0_g*16, nb1_g*16)`` of ``out`` [M, N]."""
    G, M, cols = gathered.shape
    if all((b - a) * 16 == cols for a, b in ranges) and out.is_contiguous():
        out.view(M, G, cols).copy_(gathered.permute(1, 0, 2))  # equal shards: one copy
        return out
    for g, (a, b) in enumerate(ranges):
        if b > a:
            out[:, a * 16:b * 16] = gathered[g, :, :(b - a) * 16]
    return out


def _device_gemm(sh: "ColumnShardedGemm", M, A, a_scale, C):
    from . import device as D
    if sh.cols == 0:
        return
    if sh.kind == "q4g":
        D.gemm_q4g(M, sh.cols, sh.K, A, a_scale, sh.w, sh.s, sh.group, C, ldc=sh.max_cols)
    else:
        D.gemm_q8c(M, sh.cols, sh.K, A, a_scale, sh.w, sh.s, C, ldc=sh.max_cols)


class ColumnShardedGemm:
    """One rank's share of a column-sharded q4g / q8c GEMM.

    ``blob``/``scale`` are the full host weight (numpy, .fgm layout); only
    this rank's slice is kept (on ``device``).  ``shard=(w, s)`` passes that
    slice directly (device tensors) instead.  ``gemm(shard, M, A, a_scale,
    C)`` computes the local block into C [M, max_cols]; by default it is the
    library's device GEMM on the shard.
    """

    def __init__(self, kind: str, blob: np.ndarray | None, scale: np.ndarray | None, N: int,
                 K: int, group: int = 64, *, rank: int | None = None, world: int | None = None,
                 pg=None, device=None, gemm: Callable | None = None, shard=None):
        if kind not in ("q4g", "q8c"):
            raise ValueError(f"kind must be q4g or q8c, not {kind!r}")
        self.kind, self.N, self.K, self.group, self.pg = kind, N, K, group, pg
        self.world = world if world is not None else (dist.get_world_size(pg) if dist.is_initialized() else 1)
        self.rank = rank if rank is not None else (dist.get_rank(pg) if dist.is_initialized() else 0)
        self.device = torch.device(device) if device is not None else torch.device("cpu")
        self.ranges = shard_ranges(N // 16, self.world)
        self.nb0, self.nb1 = self.ranges[self.rank]
        self.cols = (self.nb1 - self.nb0) * 16
        self.max_cols = max((b - a) * 16 for a, b in self.ranges)
        if shard is not None:  # this rank's slice, already resident: (weight, scales)
            self.w, self.s = shard
        else:
            if kind == "q4g":
                w, s = F.q4g_column_shard(blob, scale, N, K, self.nb0, self.nb1)
                s = s.view(np.uint16)
            else:
                w, s = F.q8c_column_shard(blob, scale, N, K, self.nb0, self.nb1)
            self.w = torch.from_numpy(np.ascontiguousarray(w)).to(self.device)
            self.s = torch.from_numpy(np.ascontiguousarray(s)).to(self.device)
        self._gemm = gemm or _device_gemm
        self._local = None
        self._gathered = None

    def local(self, M: int, A, a_scale) -> torch.Tensor:
        """This rank's columns, [M, max_cols] (columns past ``cols`` unused)."""
        if self._local is None or self._local.shape[0] != M:
            self._local = torch.zeros((M, self.max_cols), dtype=torch.float32, device=self.device)
        self._gemm(self, M, A, a_scale, self._local)
        return self._local

    def gather(self, local: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """All-gather every rank's block and assemble the full [M, N] output."""
        M = local.shape[0]
        if out is None:
            out = torch.empty((M, self.N), dtype=torch.float32, device=local.device)
        if self.world == 1:
            return assemble(local.unsqueeze(0), self.ranges, out)
        if self._gathered is None or self._gathered.shape[1] != M:
            self._gathered = torch.empty((self.world, M, self.max_cols), dtype=torch.float32,
                                         device=local.device)
        if local.is_cuda:
            dist.all_gather_into_tensor(self._gathered, local.contiguous(), group=self.pg)
        else:
            dist.all_gather(list(self._gathered.unbind(0)), local.contiguous(), group=self.pg)
        return assemble(self._gathered, self.ranges, out)

    def __call__(self, M: int, A, a_scale, out: torch.Tensor | None = None) -> torch.Tensor:
        if self.world == 1 and (out is None or out.is_contiguous()):  # the whole GEMM, in place
            if out is None:
                out = torch.empty((M, self.N), dtype=torch.float32, device=self.device)
            self._gemm(self, M, A, a_scale, out)
            return out
        return self.gather(self.local(M, A, a_scale), out)
