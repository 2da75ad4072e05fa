"""Device-resident entry points (include/fgm_cuda.h, "device pointers").

Every buffer is a CUDA tensor on the current device; work is enqueued on the
current torch stream (or ``stream=``) and nothing waits.  torch is used only
for allocation and stream handles; the arithmetic is the library's.
"""
from __future__ import annotations

import ctypes as C

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


# ------------------------------------------- decode-chain glue, attention
def rmsnorm(out, x, w, rows, n, eps, stream=None):
    """ops.c:59-92 over rows of n (w None: the no-scale form)."""
    call("fgm_cuda_rmsnorm", _p(out), _p(x), _p(w), rows, n, eps, _s(stream))


def gelu_mul(out, gate, up, rows, n, stream=None):
    """ops.c:119-131: out = gelu_tanh(gate) * up."""
    call("fgm_cuda_gelu_mul", _p(out), _p(gate), _p(up), rows, n, _s(stream))


def add(a, b, stream=None):
    call("fgm_cuda_add", _p(a), _p(b), a.numel(), _s(stream))


def mul(a, b, stream=None):
    call("fgm_cuda_mul", _p(a), _p(b), a.numel(), _s(stream))


def scale(a, s, stream=None):
    call("fgm_cuda_scale", _p(a), s, a.numel(), _s(stream))


def softcap(x, rows, n, cap, stream=None):
    call("fgm_cuda_softcap", _p(x), rows, n, cap, _s(stream))


def rope(x, x_ld, rows, n_heads, head_dim, inv_freq, pos, cs=None, stream=None):
    """ops.c:135-147 in place; pos: int32 device tensor [rows]; cs: a device
    copy of rope_table(...) (the reference's libm cos / sin), else the device
    evaluates them."""
    if cs is None:
        call("fgm_cuda_rope", _p(x), x_ld, rows, n_heads, head_dim, _p(inv_freq), _p(pos),
             _s(stream))
    else:
        call("fgm_cuda_rope_cs", _p(x), x_ld, rows, n_heads, head_dim, _p(inv_freq), _p(cs),
             cs.shape[0], _p(pos), _s(stream))


def rope_table(positions, head_dim, inv_freq):
    """Host [positions][head_dim] f32: cosf | sinf of (float)p * inv_freq[j]
    (ops.c:137-139) from this host's libm; inv_freq: numpy f32 [head_dim/2]."""
    import numpy as np
    inv = np.ascontiguousarray(inv_freq, dtype=np.float32)
    out = np.empty((positions, head_dim), np.float32)
    call("fgm_cuda_rope_table", out.ctypes.data, positions, head_dim, inv.ctypes.data)
    return out


def quant_act(x, rows, k, q, scale, stream=None):
    """ops.c:181-204 (quant_kv: one row)."""
    call("fgm_cuda_quant_act", _p(x), rows, k, _p(q), _p(scale), _s(stream))


def store_v_t(vt, vt_stride, src, src_ld, rows, n, slot, stream=None):
    """ops.c:653-660 for `rows` caches."""
    call("fgm_cuda_store_v_t", _p(vt), vt_stride, _p(src), src_ld, rows, n, slot, _s(stream))


def attend_q8(out, out_ld, q, q_ld, kc, kc_stride, ks, ks_stride, vt, vt_stride, vs, vs_stride,
              rows, n_heads, kv_heads, head_dim, start, end, ring=0, stream=None):
    """ops.c:378-640 for `rows` query rows, each against its own int8 KV cache."""
    call("fgm_cuda_attend_q8", _p(out), out_ld, _p(q), q_ld, _p(kc), kc_stride, _p(ks), ks_stride,
         _p(vt), vt_stride, _p(vs), vs_stride, rows, n_heads, kv_heads, head_dim, start, end, ring,
         _s(stream))


def norm_prep(h, proj, w_post, w_pre, rows, n, eps, qs, pa, stream=None):
    """forward.rs:476-480, :625-654: h += rmsnorm(proj, w_post) (when proj is
    given), then the packed rows of rmsnorm(h, w_pre)."""
    call("fgm_cuda_norm_prep", _p(h), _p(proj), _p(w_post), _p(w_pre), rows, n, eps, _p(qs), _p(pa),
         _s(stream))


def gelu_mul_prep(gate, up, rows, n, qs, pa, act=None, ld=None, stream=None):
    """forward.rs:641-643: packed rows of gelu(gate) * up (rows ld apart)."""
    call("fgm_cuda_gelu_mul_prep", _p(gate), _p(up), n if ld is None else ld, rows, n, _p(act),
         _p(qs), _p(pa), _s(stream))


def qkv_post(q, k, v, rows, n_heads, kv_heads, head_dim, q_norm, k_norm, eps, inv_freq, pos, ring,
             cap, kc, kc_stride, ks, ks_stride, vt, vt_stride, vs, vs_stride, q_ld=None, kv_ld=None,
             cs=None, stream=None):
    """forward.rs:482-545: head norms, rope, int8 K / V rows into the caches
    (cs: a device copy of rope_table(...), as for rope)."""
    q_ld = n_heads * head_dim if q_ld is None else q_ld
    kv_ld = kv_heads * head_dim if kv_ld is None else kv_ld
    call("fgm_cuda_qkv_post_cs", _p(q), q_ld, _p(k), _p(v), kv_ld, rows, n_heads, kv_heads,
         head_dim, _p(q_norm), _p(k_norm), eps, _p(inv_freq), _p(cs),
         0 if cs is None else cs.shape[0], _p(pos), ring, cap, _p(kc), kc_stride, _p(ks),
         ks_stride, _p(vt), vt_stride, _p(vs), vs_stride, _s(stream))



# ------------------------------------------------------- decode work list
class _Work(C.Structure):
    """fgm_cuda_work (include/fgm_cuda.h)."""
    _fields_ = [("kind", C.c_int), ("N", C.c_int), ("K", C.c_int), ("group", C.c_int),
                ("n0", C.c_int), ("n1", C.c_int), ("ldc", C.c_int), ("lda", C.c_int),
                ("hsz", C.c_int), ("deps", C.c_int * 2),
                ("A", C.c_void_p), ("a_scale", C.c_void_p), ("B", C.c_void_p),
                ("b_scale", C.c_void_p), ("C", C.c_void_p), ("src", C.c_void_p),
                ("pa", C.c_void_p), ("qs", C.c_void_p)]


WORK_Q4G, WORK_Q8C, WORK_PREP = 0, 1, 2


class WorkList:
    """A decode step's projections as one persistent launch
    (fgm_cuda_worklist_*).  Add entries in an order where every entry's
    dependencies come first, then ``build(M)`` once and ``run()`` per step.
    The tensors passed in must stay alive (and in place) as long as the list."""

    def __init__(self):
        self._items, self._keep, self.handle = [], [], None

    def _add(self, w, deps, keep):
        d = list(deps) + [-1, -1]
        w.deps[0], w.deps[1] = d[0], d[1]
        self._items.append(w)
        self._keep.extend(keep)
        return len(self._items) - 1

    def prep(self, src, lda, K, pa, qs, hsz=0, deps=()):
        """Rows [0, M) of src (f32) -> packed pa and scales qs (fgm_prep_rows)."""
        w = _Work(kind=WORK_PREP, K=K, lda=lda, hsz=hsz, src=_p(src), pa=_p(pa), qs=_p(qs))
        return self._add(w, deps, (src, pa, qs))

    def gemm_q4g(self, N, K, A, a_scale, Bq, b_scale, group, C, ldc=None, n0=0, n1=None,
                 deps=()):
        n1 = N // 16 if n1 is None else n1
        w = _Work(kind=WORK_Q4G, N=N, K=K, group=group, n0=n0, n1=n1,
                  ldc=N if ldc is None else ldc, A=_p(A), a_scale=_p(a_scale), B=_p(Bq),
                  b_scale=_p(b_scale), C=_p(C))
        return self._add(w, deps, (A, a_scale, Bq, b_scale, C))

    def gemm_q8c(self, N, K, A, a_scale, B, b_scale, C, ldc=None, n0=0, n1=None, deps=()):
        n1 = N // 16 if n1 is None else n1
        w = _Work(kind=WORK_Q8C, N=N, K=K, n0=n0, n1=n1, ldc=N if ldc is None else ldc,
                  A=_p(A), a_scale=_p(a_scale), B=_p(B), b_scale=_p(b_scale), C=_p(C))
        return self._add(w, deps, (A, a_scale, B, b_scale, C))

    def build(self, M):
        arr = (_Work * len(self._items))(*self._items)
        h = C.c_void_p()
        call("fgm_cuda_worklist_create", M, arr, len(self._items), C.byref(h))
        self.handle = h
        return self

    def run(self, stream=None):
        call("fgm_cuda_worklist_run", self.handle, _s(stream))

    def close(self):
        if self.handle is not None:
            call("fgm_cuda_worklist_destroy", self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
