"""fastgemma_b200 -- the sm_100a backend of fastgemma's quantised GEMM path.

Host-side mirror of ``crates/fgm-kernels/src/lib.rs`` for the GEMM path, with
the same names, argument meaning and shape contract, backed by
``libfgm_cuda.so`` (include/fgm_cuda.h):

* :func:`backend`        -- lib.rs:112-138, extended with ``Backend.CUDA``
* :func:`packed_a_len`   -- lib.rs:155-157
* :func:`pack_a`         -- lib.rs:160-164
* :func:`gemm_q4g`       -- lib.rs:171-194
* :func:`gemm_q8c`       -- lib.rs:197-217
* :func:`prep_rows`      -- lib.rs:517-530
* :func:`quant_act`, :func:`fwht` -- lib.rs:238-250

These take host (numpy) buffers like the reference's slices.  Where the
reference only debug-asserts a shape (lib.rs:177-178, :203-204) these raise
:class:`FgmCudaError` with the library's message.  Device-resident variants
for a GPU-resident caller live in :mod:`fastgemma_b200.device`.
"""
from __future__ import annotations

import enum
import os

import numpy as np

from ._lib import FgmCudaError, call, lib  # noqa: F401
from .fgm_format import packed_a_len  # noqa: F401

__all__ = ["Backend", "backend", "packed_a_len", "pack_a", "gemm_q4g", "gemm_q8c",
           "linear_q4g", "linear_q8c", "prep_rows", "quant_act", "fwht", "register",
           "unregister", "FgmCudaError"]


class Backend(enum.Enum):
    """lib.rs:86-99 plus the CUDA backend this package provides."""
    AMX = "amx"
    VNNI = "avx512-vnni"
    CUDA = "cuda"


def backend() -> Backend:
    """The GEMM backend for this process (lib.rs:112-138).

    ``FGM_BACKEND=cuda`` (or unset, when an sm_100 device is visible) selects
    CUDA.  ``amx``/``vnni`` name the reference's CPU kernels, which live in
    fgm-kernels itself and are not part of this package: asking for them here
    raises, as lib.rs:121 does for a CPU without AMX.
    """
    want = os.environ.get("FGM_BACKEND", "")
    if want in ("amx", "vnni"):
        raise RuntimeError(f"FGM_BACKEND={want}: the CPU kernels are fgm-kernels' own, "
                           "not part of fastgemma_b200")
    if not lib().fgm_cuda_available():
        raise RuntimeError("FGM_BACKEND=cuda but no sm_100 device is visible")
    return Backend.CUDA


def _p(x):
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if isinstance(x, np.ndarray):
        return x.ctypes.data
    return x.data_ptr()  # torch tensor


def _need(a: np.ndarray, dtype, name: str):
    if not isinstance(a, np.ndarray) or a.dtype != np.dtype(dtype) or not a.flags.c_contiguous:
        raise TypeError(f"{name} must be a C-contiguous numpy array of {np.dtype(dtype)}")


def pack_a(m: int, k: int, a: np.ndarray, ap: np.ndarray) -> None:
    """Tile-pack ``a[m, k]`` int8 into ``ap`` (lib.rs:160-164)."""
    _need(a, np.int8, "a")
    _need(ap, np.int8, "ap")
    if a.size < m * k or ap.size < packed_a_len(m, k):
        raise ValueError("pack_a: buffer too small")
    call("fgm_pack_a_cuda", m, k, _p(a), _p(ap))


def gemm_q4g(m, n, k, a, a_scale, bq, b_scale, group, c, ldc, n0, n1) -> None:
    """``C[m, n] = (A int8 * a_scale) . (int4-grouped B * b_scale)`` for
    columns ``[n0*16, n1*16)``; ``a`` tile-packed (lib.rs:171-194)."""
    _need(a, np.int8, "a")
    _need(bq, np.uint8, "bq")
    _need(c, np.float32, "c")
    if a.size < packed_a_len(m, k) or bq.size < n * k // 2 or c.size < max(m - 1, 0) * ldc + n:
        raise ValueError("gemm_q4g: buffer too small")
    call("fgm_gemm_q4g_cuda", m, n, k, _p(a), _p(a_scale), _p(bq),
         _p(np.ascontiguousarray(b_scale).view(np.uint16)), group, _p(c), ldc, n0, n1)


def gemm_q8c(m, n, k, a, a_scale, b, b_scale, c, ldc, n0, n1) -> None:
    """``C[m, n] = (A int8 * a_scale) . (int8 per-channel B * b_scale)``
    (lib.rs:197-217)."""
    _need(a, np.int8, "a")
    _need(b, np.int8, "b")
    _need(c, np.float32, "c")
    if a.size < packed_a_len(m, k) or b.size < n * k or c.size < max(m - 1, 0) * ldc + n:
        raise ValueError("gemm_q8c: buffer too small")
    call("fgm_gemm_q8c_cuda", m, n, k, _p(a), _p(a_scale), _p(b), _p(b_scale), _p(c), ldc,
         n0, n1)


def linear_q4g(src, lda, hsz, m, n, k, bq, b_scale, group, c, ldc) -> None:
    """``Gemm::run`` for an int4 weight (forward.rs:128-158): rotate, quantise
    and pack ``src[m, lda]`` on the device, then the GEMM over all columns."""
    call("fgm_linear_q4g_cuda", _p(src), lda, hsz, m, n, k, _p(bq),
         _p(np.ascontiguousarray(b_scale).view(np.uint16)), group, _p(c), ldc)


def linear_q8c(src, lda, hsz, m, n, k, b, b_scale, c, ldc) -> None:
    """``Gemm::run`` for an int8 weight (forward.rs:128-158)."""
    call("fgm_linear_q8c_cuda", _p(src), lda, hsz, m, n, k, _p(b), _p(b_scale), _p(c), ldc)


def prep_rows(src, lda, rot, qa, qs, pa, m, k, hsz, r0, r1) -> None:
    """Rotate + quantise + tile-pack rows ``[r0, r1)`` (lib.rs:517-530)."""
    if r0 % 16:
        raise ValueError("prep row start must be tile-aligned")
    call("fgm_prep_rows_cuda", _p(src), lda, _p(rot), _p(qa), _p(qs), _p(pa), m, k, hsz, r0, r1)


def quant_act(x, rows, k, q, scale) -> None:
    """Per-row symmetric int8 quantisation (lib.rs:238-240)."""
    call("fgm_quant_act_cuda", _p(x), rows, k, _p(q), _p(scale))


def fwht(x: np.ndarray, hsz: int) -> None:
    """In-place normalised FWHT on blocks of ``hsz`` (lib.rs:231-236)."""
    _need(x, np.float32, "x")
    call("fgm_fwht_cuda", _p(x), x.size, hsz)


def register(host: np.ndarray) -> None:
    """Upload an immutable weight blob once; later calls resolve it by address."""
    call("fgm_cuda_register", _p(host), host.nbytes)


def unregister(host: np.ndarray) -> None:
    call("fgm_cuda_unregister", _p(host))
