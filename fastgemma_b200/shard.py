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
same X.  The full output is assembled either with one all-gather of the
per-rank column blocks over the process group (NCCL over NVLink on GPUs,
gloo on CPU), or -- ``fused=True``, the int4 decode GEMM -- inside the GEMM
kernel itself: each rank's finished columns are stored straight into every
peer's output over NVLink (CUDA IPC buffers, system-scope counters), one
kernel per rank and no separate collective.

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


class _DeviceArray:
    """A raw device allocation seen by torch without a copy."""

    def __init__(self, ptr: int, shape, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (ptr, False), "version": 3, "strides": None}


SIG_BYTES = 128  # FGM_CUDA_GATHER_SIG_BYTES


class PeerBuffers:
    """Every rank's double-buffered output [2][rows][N] f32 and signal words,
    allocated by the owner and opened by every peer (CUDA IPC, one node).
    Collective: all ranks of the group construct it together."""

    def __init__(self, rows: int, N: int, rank: int, world: int, pg=None):
        import ctypes as C
        from ._lib import call, lib
        self.rows, self.N, self.rank, self.world = rows, N, rank, world
        self.slot_bytes = rows * N * 4
        out, sig = C.c_void_p(), C.c_void_p()
        call("fgm_cuda_ipc_alloc", 2 * self.slot_bytes, C.byref(out))
        call("fgm_cuda_ipc_alloc", SIG_BYTES, C.byref(sig))
        self._own = (out.value, sig.value)
        h_out, h_sig = (C.c_ubyte * 64)(), (C.c_ubyte * 64)()
        call("fgm_cuda_ipc_handle", out, h_out)
        call("fgm_cuda_ipc_handle", sig, h_sig)
        handles = [None] * world
        mine = (bytes(h_out), bytes(h_sig))
        if world > 1:
            dist.all_gather_object(handles, mine, group=pg)
        else:
            handles = [mine]
        self.out, self.sig, self._opened = [], [], []
        for q, (ho, hs) in enumerate(handles):
            if q == rank:
                self.out.append(out.value)
                self.sig.append(sig.value)
                continue
            po, ps = C.c_void_p(), C.c_void_p()
            call("fgm_cuda_ipc_open", (C.c_ubyte * 64).from_buffer_copy(ho), C.byref(po))
            call("fgm_cuda_ipc_open", (C.c_ubyte * 64).from_buffer_copy(hs), C.byref(ps))
            self.out.append(po.value)
            self.sig.append(ps.value)
            self._opened += [po.value, ps.value]
        self._lib = lib()

    def view(self, slot: int, M: int, device) -> torch.Tensor:
        ptr = self.out[self.rank] + slot * self.slot_bytes
        return torch.as_tensor(_DeviceArray(ptr, (self.rows, self.N)), device=device)[:M]

    def stamps(self, device) -> dict:
        """%globaltimer stamps (ns) of this rank's last fused call: start, own
        columns pushed, every rank's columns arrived; and its completed calls."""
        w = torch.as_tensor(_DeviceArray(self.sig[self.rank], (SIG_BYTES // 8,), "<u8"),
                            device=device).cpu().numpy()
        return {"calls": int(w[6]), "start": int(w[8]), "pushed": int(w[9]),
                "arrived": int(w[10])}

    def close(self):
        from ._lib import call
        for p in self._opened:
            call("fgm_cuda_ipc_close", p)
        self._opened = []
        for p in self._own:
            call("fgm_cuda_ipc_free", p)
        self._own = ()


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
                 pg=None, device=None, gemm: Callable | None = None, shard=None,
                 fused: bool = False, max_rows: int = 16):
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
        # fused: one kernel per call computes this rank's columns and stores
        # them into every rank's output over NVLink (int4 decode GEMM only)
        self.peers = None
        self._calls = 0
        self._args = None
        if fused:
            if kind != "q4g" or max_rows > 16:
                raise ValueError("the fused gather covers the int4 decode GEMM (M <= 16)")
            self.peers = PeerBuffers(max_rows, N, self.rank, self.world, pg)

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

    def fused_call(self, M: int, A, a_scale, stream=None) -> torch.Tensor:
        """GEMM + all-gather in one kernel per rank; returns this rank's view
        of the full [M, N] output (valid until the call after next)."""
        import ctypes as C
        from ._lib import call
        pb = self.peers
        if M > pb.rows:
            raise ValueError(f"M={M} > max_rows={pb.rows}")
        slot = self._calls & 1  # the kernel counts the calls itself; this only picks the view
        self._calls += 1
        if self._args is None:
            self._args = ((C.c_void_p * self.world)(*pb.out), (C.c_void_p * self.world)(*pb.sig))
        outs, sigs = self._args
        st = (stream or torch.cuda.current_stream(self.device)).cuda_stream
        A_p = A.data_ptr() if hasattr(A, "data_ptr") else A
        s_p = a_scale.data_ptr() if hasattr(a_scale, "data_ptr") else a_scale
        call("fgm_cuda_gemm_q4g_gather", M, self.cols, self.K, A_p, s_p, self.w.data_ptr(),
             self.s.data_ptr(), self.group, self.nb0 * 16, self.N, outs, sigs, self.rank,
             self.world, pb.slot_bytes // 4, st)
        return pb.view(slot, M, self.device)

    def argmax(self, M: int, A, a_scale, stream=None) -> torch.Tensor:
        """Token choice for each row (engine.rs:75-83).  With peer buffers
        (fused=True, several ranks) the fused GEMM + all-gather kernel already
        leaves every rank the whole logits matrix, so each rank scans it on
        device.  Otherwise this rank's columns reduce to per-row (value,
        index) pairs, the ranks exchange those pairs (not the logits), and
        the pairs merge into int32 [M]."""
        from ._lib import call, lib
        st = (stream or torch.cuda.current_stream(self.device)).cuda_stream
        if self.peers is not None and self.world > 1:
            logits = self.fused_call(M, A, a_scale, stream)
            parts = lib().fgm_cuda_argmax_parts(self.N)
            vals = torch.empty((M, parts), dtype=torch.float32, device=self.device)
            idx = torch.empty((M, parts), dtype=torch.int32, device=self.device)
            call("fgm_cuda_argmax_partials", logits.data_ptr(), M, self.N, self.N, 0,
                 vals.data_ptr(), idx.data_ptr(), st)
            out = torch.empty(M, dtype=torch.int32, device=self.device)
            call("fgm_cuda_argmax_merge", vals.data_ptr(), idx.data_ptr(), M, parts,
                 out.data_ptr(), st)
            return out
        local = self.local(M, A, a_scale)
        parts = lib().fgm_cuda_argmax_parts(self.max_cols)
        vals = torch.empty((M, parts), dtype=torch.float32, device=self.device)
        idx = torch.empty((M, parts), dtype=torch.int32, device=self.device)
        call("fgm_cuda_argmax_partials", local.data_ptr(), M, self.cols, self.max_cols,
             self.nb0 * 16, vals.data_ptr(), idx.data_ptr(), st)
        if self.world > 1:
            gv = torch.empty((self.world, M, parts), dtype=torch.float32, device=self.device)
            gi = torch.empty((self.world, M, parts), dtype=torch.int32, device=self.device)
            if vals.is_cuda:
                dist.all_gather_into_tensor(gv, vals, group=self.pg)
                dist.all_gather_into_tensor(gi, idx, group=self.pg)
            vals = gv.permute(1, 0, 2).reshape(M, self.world * parts).contiguous()
            idx = gi.permute(1, 0, 2).reshape(M, self.world * parts).contiguous()
        out = torch.empty(M, dtype=torch.int32, device=self.device)
        call("fgm_cuda_argmax_merge", vals.data_ptr(), idx.data_ptr(), M, vals.shape[1],
             out.data_ptr(), st)
        return out

    def close(self):
        if self.peers is not None:
            torch.cuda.synchronize(self.device)
            self.peers.close()
            self.peers = None

    def __call__(self, M: int, A, a_scale, out: torch.Tensor | None = None) -> torch.Tensor:
        if self.peers is not None and self.world > 1:
            res = self.fused_call(M, A, a_scale)
            if out is not None:
                out.copy_(res)
                return out
            return res
        if self.world == 1 and (out is None or out.is_contiguous()):  # the whole GEMM, in place
            if out is None:
                out = torch.empty((M, self.N), dtype=torch.float32, device=self.device)
            self._gemm(self, M, A, a_scale, out)
            return out
        return self.gather(self.local(M, A, a_scale), out)
