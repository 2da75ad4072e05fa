"""Device-resident entry points (include/fgm_cuda.h, "device pointers").

Every buffer is a CUDA tensor on the current device; work is enqueued on the
current torch stream (or ``stream=``) and nothing waits.  torch is used only
for allocation and stream handles; the arithmetic is the library's.
"""
from __future__ import annotations

import torch

from ._lib import call


def _s(stream):
    return (stream or torch.cuda.current_stream()).cuda_stream


def _p(t):
    return None if t is None else t.data_ptr()


def gemm_q4g(M, N, K, A, a_scale, Bq, b_scale, group, C, ldc=None, n0=0, n1=None, stream=None):
    n1 = N // 16 if n1 is None else n1
    call("fgm_cuda_gemm_q4g", M, N, K, _p(A), _p(a_scale), _p(Bq), _p(b_scale), group, _p(C),
         N if ldc is None else ldc, n0, n1, _s(stream))


def gemm_q8c(M, N, K, A, a_scale, B, b_scale, C, ldc=None, n0=0, n1=None, stream=None):
    n1 = N // 16 if n1 is None else n1
    call("fgm_cuda_gemm_q8c", M, N, K, _p(A), _p(a_scale), _p(B), _p(b_scale), _p(C),
         N if ldc is None else ldc, n0, n1, _s(stream))


def _warm_args(warm):
    """(weights, scales) tensors of the next launch -> the four warm arguments."""
    w, s = (tuple(warm) + (None, None))[:2] if warm is not None else (None, None)
    nbytes = lambda t: 0 if t is None else t.numel() * t.element_size()
    return _p(w), nbytes(w), _p(s), nbytes(s)


def gemm_q4g_warm(M, N, K, A, a_scale, Bq, b_scale, group, C, warm, ldc=None, n0=0, n1=None,
                  stream=None):
    """gemm_q4g that also prefetches warm = (next weights, next scales) into L2."""
    n1 = N // 16 if n1 is None else n1
    call("fgm_cuda_gemm_q4g_warm", M, N, K, _p(A), _p(a_scale), _p(Bq), _p(b_scale), group,
         _p(C), N if ldc is None else ldc, n0, n1, *_warm_args(warm), _s(stream))


def gemm_q8c_warm(M, N, K, A, a_scale, B, b_scale, C, warm, ldc=None, n0=0, n1=None,
                  stream=None):
    """gemm_q8c that also prefetches warm = (next weights, next scales) into L2."""
    n1 = N // 16 if n1 is None else n1
    call("fgm_cuda_gemm_q8c_warm", M, N, K, _p(A), _p(a_scale), _p(B), _p(b_scale), _p(C),
         N if ldc is None else ldc, n0, n1, *_warm_args(warm), _s(stream))


def gemm_q4g_acc(M, N, K, A, Bq, group, acc, n0=0, n1=None, stream=None):
    n1 = N // 16 if n1 is None else n1
    call("fgm_cuda_gemm_q4g_acc", M, N, K, _p(A), _p(Bq), group, _p(acc), n0, n1, _s(stream))


def gemm_q8c_acc(M, N, K, A, B, acc, n0=0, n1=None, stream=None):
    n1 = N // 16 if n1 is None else n1
    call("fgm_cuda_gemm_q8c_acc", M, N, K, _p(A), _p(B), _p(acc), n0, n1, _s(stream))


def prep_rows(src, lda, qs, pa, m, k, hsz, rot=None, qa=None, r0=0, r1=None, stream=None):
    r1 = m if r1 is None else r1
    call("fgm_cuda_prep_rows", _p(src), lda, _p(rot), _p(qa), _p(qs), _p(pa), m, k, hsz, r0, r1,
         _s(stream))


def linear_q4g(src, lda, hsz, M, N, K, Bq, b_scale, group, C, ldc=None, n0=0, n1=None,
               stream=None):
    """Gemm::run for one int4 projection: f32 rows in, C out (prep fused for M <= 16)."""
    n1 = N // 16 if n1 is None else n1
    call("fgm_cuda_linear_q4g", _p(src), lda, hsz, M, N, K, _p(Bq), _p(b_scale), group, _p(C),
         N if ldc is None else ldc, n0, n1, _s(stream))


def linear_q8c(src, lda, hsz, M, N, K, B, b_scale, C, ldc=None, n0=0, n1=None, stream=None):
    """Gemm::run for one int8 projection (tensor cores for prepared weights, M >= 64)."""
    n1 = N // 16 if n1 is None else n1
    call("fgm_cuda_linear_q8c", _p(src), lda, hsz, M, N, K, _p(B), _p(b_scale), _p(C),
         N if ldc is None else ldc, n0, n1, _s(stream))


def packed_a(m: int, k: int, device=None) -> torch.Tensor:
    """An uninitialised packed-activation buffer of ``packed_a_len(m, k)`` bytes."""
    return torch.empty((m + 15) // 16 * 16 * k, dtype=torch.int8, device=device or "cuda")


def gemm_q8c_rows(M, N, K, A, a_scale, B, b_scale, C, lda=None, ldc=None, n0=0, n1=None,
                  stream=None):
    """Prefill int8 GEMM from row-major int8 activations (prepared weight)."""
    n1 = N // 16 if n1 is None else n1
    call("fgm_cuda_gemm_q8c_rows", M, N, K, _p(A), K if lda is None else lda, _p(a_scale), _p(B),
         _p(b_scale), _p(C), N if ldc is None else ldc, n0, n1, _s(stream))


def gemm_q8c_noalloc(M, N, K, A, a_scale, B, b_scale, C, ldc=None, n0=0, n1=None, stream=None):
    """gemm_q8c on the tensor-core kernel with no device allocation (prepared
    weight, M*K <= 4 MiB; concurrent calls on one device race)."""
    n1 = N // 16 if n1 is None else n1
    call("fgm_cuda_gemm_q8c_noalloc", M, N, K, _p(A), _p(a_scale), _p(B), _p(b_scale), _p(C),
         N if ldc is None else ldc, n0, n1, _s(stream))


def q8c_prepare(B, N, K, stream=None):
    """Make the tensor-core operand copy of a device int8 weight (large-M path)."""
    call("fgm_cuda_q8c_prepare", _p(B), N, K, _s(stream))


def q8c_release(B):
    call("fgm_cuda_q8c_release", _p(B))
