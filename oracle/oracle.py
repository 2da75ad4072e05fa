"""ctypes front-end to the parity checkers.  TEST INFRASTRUCTURE ONLY.

Two libraries, both built by ``oracle/Makefile``:

* ``liboracle.so`` -- ``fgm_oracle.c``, the scalar C restatement of the
  reference algorithm (always buildable with gcc), plus the pool driver.
* ``_ref/libfgm_ref.so`` -- the reference's own kernels
  (``crates/fgm-kernels/csrc/{amx_gemm,vnni_gemm,ops}.c``) compiled from their
  sources, plus the same pool driver.  Present only where the reference tree
  was available at build time.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg import this module.  The shipped library never does.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libfgm_ref.so")

_p = C.c_void_p
_i = C.c_int


def _ptr(a):
    return a.ctypes.data_as(_p) if a is not None else None


def _decl(lib, name, argtypes, restype=None):
    f = getattr(lib, name)
    f.argtypes = argtypes
    f.restype = restype
    return f


_GEMM_Q4G = [_i, _i, _i, _p, _p, _p, _p, _i, _p, _i, _i, _i]
_GEMM_Q8C = [_i, _i, _i, _p, _p, _p, _p, _p, _i, _i, _i]
_PREP = [_p, _i, _p, _p, _p, _p, _i, _i, _i, _i, _i]
_POOL = {
    "cpu_pool_start": ([_i, _p], _i),
    "cpu_pool_stop": ([], None),
    "cpu_pool_threads": ([], _i),
    "cpu_pool_gemm_q4g": ([_p, _i, _i, _i, _p, _p, _p, _p, _i, _p, _i], None),
    "cpu_pool_gemm_q8c": ([_p, _i, _i, _i, _p, _p, _p, _p, _p, _i], None),
    "cpu_pool_prep": ([_p, _p, _i, _p, _p, _p, _p, _i, _i, _i], None),
    "cpu_pool_now": ([], C.c_double),
}


def _load_pool(lib):
    for name, (args, res) in _POOL.items():
        _decl(lib, name, args, res)


class _Glue:
    """The decode-chain glue and attention, same methods on both libraries
    (prefix ``orc_`` for the restatement, ``fgm_`` for the reference)."""

    prefix = ""

    def _f(self, name):
        return getattr(self.lib, self.prefix + name)

    def rmsnorm(self, x, w, eps):
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty_like(x)
        n = x.shape[-1]
        for r in range(x.size // n):
            xo, oo = x.reshape(-1, n)[r], out.reshape(-1, n)[r]
            if w is None:
                self._f("rmsnorm_noscale")(_ptr(oo), _ptr(xo), n, C.c_float(eps)) \
                    if self.prefix == "fgm_" else \
                    self._f("rmsnorm")(_ptr(oo), _ptr(xo), None, n, C.c_float(eps))
            else:
                self._f("rmsnorm")(_ptr(oo), _ptr(xo), _ptr(np.ascontiguousarray(w, np.float32)),
                                   n, C.c_float(eps))
        return out

    def gelu_mul(self, gate, up):
        gate = np.ascontiguousarray(gate, np.float32)
        up = np.ascontiguousarray(up, np.float32)
        out = np.empty_like(gate)
        self._f("gelu_mul")(_ptr(out), _ptr(gate), _ptr(up), gate.size)
        return out

    def add(self, a, b):
        a = np.ascontiguousarray(a, np.float32).copy()
        self._f("add")(_ptr(a), _ptr(np.ascontiguousarray(b, np.float32)), a.size)
        return a

    def softcap(self, x, cap):
        x = np.ascontiguousarray(x, np.float32).copy()
        self._f("softcap")(_ptr(x), x.size, C.c_float(cap))
        return x

    def quant_act(self, x: np.ndarray):
        """ops.c:181-204: rows to int8 with one scale each."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        rows, k = x.shape
        q = np.empty((rows, k), np.int8)
        s = np.empty(rows, np.float32)
        self._f("quant_act")(_ptr(x), rows, k, _ptr(q), _ptr(s))
        return q, s

    def store_v_t(self, vt, src, slot):
        src = np.ascontiguousarray(src, np.int8)
        self._f("store_v_t")(_ptr(vt), _ptr(src), src.size, slot)

    def attend_q8(self, q, kc, ks, vc, vs, n_heads, kv_heads, head_dim, start, end, ring=0):
        q = np.ascontiguousarray(q, np.float32)
        out = np.zeros(n_heads * head_dim, np.float32)
        cap = max(end, ring, 1)
        scratch = np.zeros(2 * cap + 2 * head_dim + 64, np.float32)
        args = [_ptr(out), _ptr(q), _ptr(kc), _ptr(ks), _ptr(vc), _ptr(vs), n_heads, kv_heads,
                head_dim, start, end, _ptr(scratch), 0, n_heads, ring]
        if self.prefix == "fgm_":
            args.append(cap)
        self._f("attend_q8_heads")(*args)
        return out


class Oracle(_Glue):
    """The scalar C restatement (``fgm_oracle.c``)."""

    prefix = "orc_"

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle`")
        self.lib = C.CDLL(path)
        L = self.lib
        _decl(L, "orc_f16_to_f32", [C.c_uint16], C.c_float)
        _decl(L, "orc_nibble", [_i], _i)
        _decl(L, "orc_cvt_sat_i8", [C.c_float], C.c_int8)
        _decl(L, "orc_fwht", [_p, _i, _i])
        _decl(L, "orc_quant_act", [_p, _i, _i, _p, _p])
        _decl(L, "orc_pack_a", [_i, _i, _p, _p])
        _decl(L, "orc_prep_rows", _PREP)
        _decl(L, "orc_gemm_q4g", _GEMM_Q4G)
        _decl(L, "orc_gemm_q4g_acc", [_i, _i, _i, _p, _p, _i, _p, _i, _i])
        _decl(L, "orc_gemm_q8c", _GEMM_Q8C)
        _decl(L, "orc_gemm_q8c_acc", [_i, _i, _i, _p, _p, _p, _i, _i])
        _decl(L, "orc_unpack_q4_tiles", [_p, C.c_size_t, _p])
        _decl(L, "orc_fill_xorshift", [_p, _i, _i, C.c_size_t, _p])
        _decl(L, "orc_fill_lcg", [_p, _i, _i, C.c_size_t, _p])
        _decl(L, "orc_argmax", [_p, _i], _i)
        _decl(L, "orc_exp_lane", [C.c_float], C.c_float)
        _decl(L, "orc_rmsnorm", [_p, _p, _p, _i, C.c_float])
        _decl(L, "orc_gelu_mul", [_p, _p, _p, _i])
        _decl(L, "orc_add", [_p, _p, _i])
        _decl(L, "orc_softcap", [_p, _i, C.c_float])
        _decl(L, "orc_rope", [_p, _i, _i, _p, _i, _i])
        _decl(L, "orc_store_v_t", [_p, _p, _i, _i])
        _decl(L, "orc_attend_q8_heads", [_p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _p, _i, _i,
                                         _i])
        _load_pool(L)
        self.kind = "port"

    def rope(self, x, n_heads, head_dim, inv_freq, pos, fused=True):
        """ops.c:135-147 as the reference build compiles it (products and sum
        fused); fused=False rounds each product."""
        x = np.ascontiguousarray(x, np.float32).copy()
        self.lib.orc_rope(_ptr(x), n_heads, head_dim,
                          _ptr(np.ascontiguousarray(inv_freq, np.float32)), pos, int(fused))
        return x

    # -- the reference harnesses' PRNGs --------------------------------------
    def xorshift(self, state: np.ndarray, lo: int, hi: int, n: int) -> np.ndarray:
        """vnni_test.c:39-43; ``state`` is a 1-element uint64 array, advanced."""
        out = np.empty(n, np.int32)
        self.lib.orc_fill_xorshift(_ptr(state), lo, hi, n, _ptr(out))
        return out

    def lcg(self, state: np.ndarray, lo: int, hi: int, n: int) -> np.ndarray:
        """gemm_test.c:30-31; ``state`` is a 1-element uint32 array, advanced."""
        out = np.empty(n, np.int32)
        self.lib.orc_fill_lcg(_ptr(state), lo, hi, n, _ptr(out))
        return out

    # -- prep ----------------------------------------------------------------
    def fwht(self, x: np.ndarray, hsz: int) -> np.ndarray:
        y = np.ascontiguousarray(x, dtype=np.float32).copy()
        self.lib.orc_fwht(_ptr(y), y.size, hsz)
        return y

    def pack_a(self, a: np.ndarray) -> np.ndarray:
        a = np.ascontiguousarray(a, dtype=np.int8)
        m, k = a.shape
        ap = np.empty(((m + 15) // 16) * 16 * k, np.int8)
        self.lib.orc_pack_a(m, k, _ptr(a), _ptr(ap))
        return ap

    def prep_rows(self, src: np.ndarray, m: int, k: int, hsz: int, lda: int | None = None):
        """Whole-matrix fgm_prep_rows: returns (rot, qa, qs, pa)."""
        lda = k if lda is None else lda
        src = np.ascontiguousarray(src, dtype=np.float32)
        rot = np.zeros((m, k), np.float32)
        qa = np.zeros((m, k), np.int8)
        qs = np.zeros(m, np.float32)
        pa = np.zeros(((m + 15) // 16) * 16 * k, np.int8)
        self.lib.orc_prep_rows(_ptr(src), lda, _ptr(rot), _ptr(qa), _ptr(qs), _ptr(pa),
                               m, k, hsz, 0, m)
        return rot, qa, qs, pa

    # -- GEMMs ---------------------------------------------------------------
    def gemm_q4g(self, M, N, K, ap, a_scale, bq, b_scale, group, c=None, ldc=None,
                 n0=0, n1=None):
        n1 = N // 16 if n1 is None else n1
        ldc = N if ldc is None else ldc
        if c is None:
            c = np.zeros((max(M, 1), ldc), np.float32)
        self.lib.orc_gemm_q4g(M, N, K, _ptr(ap), _ptr(a_scale), _ptr(bq), _ptr(b_scale),
                              group, _ptr(c), ldc, n0, n1)
        return c

    def gemm_q4g_acc(self, M, N, K, ap, bq, group, n0=0, n1=None):
        n1 = N // 16 if n1 is None else n1
        acc = np.zeros((M, K // group, N), np.int32)
        self.lib.orc_gemm_q4g_acc(M, N, K, _ptr(ap), _ptr(bq), group, _ptr(acc), n0, n1)
        return acc

    def gemm_q8c(self, M, N, K, ap, a_scale, b, b_scale, c=None, ldc=None, n0=0, n1=None):
        n1 = N // 16 if n1 is None else n1
        ldc = N if ldc is None else ldc
        if c is None:
            c = np.zeros((max(M, 1), ldc), np.float32)
        self.lib.orc_gemm_q8c(M, N, K, _ptr(ap), _ptr(a_scale), _ptr(b), _ptr(b_scale),
                              _ptr(c), ldc, n0, n1)
        return c

    def gemm_q8c_acc(self, M, N, K, ap, b, n0=0, n1=None):
        n1 = N // 16 if n1 is None else n1
        acc = np.zeros((M, N), np.int32)
        self.lib.orc_gemm_q8c_acc(M, N, K, _ptr(ap), _ptr(b), _ptr(acc), n0, n1)
        return acc

    def argmax_rows(self, c: np.ndarray) -> np.ndarray:
        """Per row of c [M, N]: the reference's argmax (engine.rs:75-83)."""
        c = np.ascontiguousarray(c, dtype=np.float32)
        return np.array([self.lib.orc_argmax(_ptr(c[m]), c.shape[1]) for m in range(c.shape[0])],
                        np.int32)

    def unpack_q4_tiles(self, bq: np.ndarray) -> np.ndarray:
        nt = bq.size // 512
        out = np.empty(nt * 1024, np.int8)
        self.lib.orc_unpack_q4_tiles(_ptr(bq), nt, _ptr(out))
        return out

    # symbols the CPU pool drives
    def fn(self, name):
        table = {"q4g": "orc_gemm_q4g", "q8c": "orc_gemm_q8c", "prep": "orc_prep_rows"}
        return C.cast(getattr(self.lib, table[name]), _p).value


class Reference(_Glue):
    """The reference kernels compiled from their own sources (``oracle/_ref``)."""

    prefix = "fgm_"

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle ref`")
        self.lib = C.CDLL(path)
        L = self.lib
        _decl(L, "fgm_cpu_has_amx", [], _i)
        _decl(L, "fgm_cpu_has_avx512_vnni", [], _i)
        _decl(L, "fgm_amx_init", [], _i)
        _decl(L, "fgm_tile_guard_set", [_i])
        for n in ("fgm_gemm_q4g", "fgm_gemm_q4g_vnni"):
            _decl(L, n, _GEMM_Q4G)
        for n in ("fgm_gemm_q8c", "fgm_gemm_q8c_vnni"):
            _decl(L, n, _GEMM_Q8C)
        _decl(L, "fgm_prep_rows", _PREP)
        _decl(L, "fgm_quant_act", [_p, _i, _i, _p, _p])
        _decl(L, "fgm_fwht", [_p, _i, _i])
        _decl(L, "fgm_pack_a", [_i, _i, _p, _p])
        _decl(L, "fgm_rmsnorm", [_p, _p, _p, _i, C.c_float])
        _decl(L, "fgm_rmsnorm_noscale", [_p, _p, _i, C.c_float])
        _decl(L, "fgm_gelu_mul", [_p, _p, _p, _i])
        _decl(L, "fgm_add", [_p, _p, _i])
        _decl(L, "fgm_softcap", [_p, _i, C.c_float])
        _decl(L, "fgm_rope", [_p, _i, _i, _p, _i])
        _decl(L, "fgm_store_v_t", [_p, _p, _i, _i])
        _decl(L, "fgm_attend_q8_heads", [_p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _p, _i, _i,
                                         _i, _i])
        _load_pool(L)
        self.has_amx = bool(L.fgm_cpu_has_amx())
        self.has_vnni = bool(L.fgm_cpu_has_avx512_vnni())
        # lib.rs:112-138: AMX when CPUID reports it and the tile grant succeeds
        self.backend = None
        if self.has_amx and L.fgm_amx_init():
            self.backend = "amx"
        elif self.has_vnni:
            self.backend = "vnni"
        self.kind = "reference"

    @property
    def usable(self) -> bool:
        return self.backend is not None

    def _gemm_name(self, base, backend=None):
        b = backend or self.backend
        if b is None:
            raise RuntimeError("host CPU has neither AMX nor AVX-512 VNNI")
        return base if b == "amx" else base + "_vnni"

    def gemm_q4g(self, M, N, K, ap, a_scale, bq, b_scale, group, c=None, ldc=None,
                 n0=0, n1=None, backend=None):
        n1 = N // 16 if n1 is None else n1
        ldc = N if ldc is None else ldc
        if c is None:
            c = np.zeros((max(M, 1), ldc), np.float32)
        getattr(self.lib, self._gemm_name("fgm_gemm_q4g", backend))(
            M, N, K, _ptr(ap), _ptr(a_scale), _ptr(bq), _ptr(b_scale), group, _ptr(c),
            ldc, n0, n1)
        return c

    def gemm_q8c(self, M, N, K, ap, a_scale, b, b_scale, c=None, ldc=None, n0=0,
                 n1=None, backend=None):
        n1 = N // 16 if n1 is None else n1
        ldc = N if ldc is None else ldc
        if c is None:
            c = np.zeros((max(M, 1), ldc), np.float32)
        getattr(self.lib, self._gemm_name("fgm_gemm_q8c", backend))(
            M, N, K, _ptr(ap), _ptr(a_scale), _ptr(b), _ptr(b_scale), _ptr(c), ldc, n0, n1)
        return c

    def prep_rows(self, src, m, k, hsz, lda=None):
        lda = k if lda is None else lda
        src = np.ascontiguousarray(src, dtype=np.float32)
        rot = np.zeros((m, k), np.float32)
        qa = np.zeros((m, k), np.int8)
        qs = np.zeros(m, np.float32)
        pa = np.zeros(((m + 15) // 16) * 16 * k, np.int8)
        self.lib.fgm_prep_rows(_ptr(src), lda, _ptr(rot), _ptr(qa), _ptr(qs), _ptr(pa),
                               m, k, hsz, 0, m)
        return rot, qa, qs, pa

    def rope(self, x, n_heads, head_dim, inv_freq, pos):
        x = np.ascontiguousarray(x, np.float32).copy()
        self.lib.fgm_rope(_ptr(x), n_heads, head_dim,
                          _ptr(np.ascontiguousarray(inv_freq, np.float32)), pos)
        return x

    def fn(self, name):
        table = {"q4g": self._gemm_name("fgm_gemm_q4g"),
                 "q8c": self._gemm_name("fgm_gemm_q8c"), "prep": "fgm_prep_rows"}
        return C.cast(getattr(self.lib, table[name]), _p).value

    def init_fn(self):
        """Per-thread init for the pool: AMX tile permission (pool.rs:242)."""
        if self.backend == "amx":
            return C.cast(self.lib.fgm_amx_init, _p).value
        return None


def load_reference():
    """The reference kernels if built and runnable on this CPU, else None."""
    try:
        r = Reference()
    except (FileNotFoundError, OSError):
        return None
    return r if r.usable else None
