"""ctypes binding of libfgm_cuda.so (include/fgm_cuda.h).

The library is the product; this module only loads it and turns negative
status codes into exceptions.  Loading fails loudly when the shared object is
missing -- there is no CPU fallback behind these functions.
"""
from __future__ import annotations

import ctypes as C
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libfgm_cuda.so")

_p, _i, _sz = C.c_void_p, C.c_int, C.c_size_t

# symbol -> (argtypes, restype); every symbol include/fgm_cuda.h declares
SIGNATURES = {
    "fgm_cuda_available": ([], _i),
    "fgm_cuda_init": ([_i], _i),
    "fgm_cuda_last_error": ([], C.c_char_p),
    "fgm_cuda_launch_count": ([], C.c_uint64),
    "fgm_cuda_device_status": ([], _i),
    "fgm_gemm_q4g_cuda": ([_i, _i, _i, _p, _p, _p, _p, _i, _p, _i, _i, _i], _i),
    "fgm_gemm_q8c_cuda": ([_i, _i, _i, _p, _p, _p, _p, _p, _i, _i, _i], _i),
    "fgm_linear_q4g_cuda": ([_p, _i, _i, _i, _i, _i, _p, _p, _i, _p, _i], _i),
    "fgm_linear_q8c_cuda": ([_p, _i, _i, _i, _i, _i, _p, _p, _p, _i], _i),
    "fgm_prep_rows_cuda": ([_p, _i, _p, _p, _p, _p, _i, _i, _i, _i, _i], _i),
    "fgm_quant_act_cuda": ([_p, _i, _i, _p, _p], _i),
    "fgm_fwht_cuda": ([_p, _i, _i], _i),
    "fgm_pack_a_cuda": ([_i, _i, _p, _p], _i),
    "fgm_cuda_register": ([_p, _sz], _i),
    "fgm_cuda_unregister": ([_p], _i),
    "fgm_cuda_lookup": ([_p], _p),
    "fgm_cuda_registry_bytes": ([], _sz),
    "fgm_cuda_gemm_q4g": ([_i, _i, _i, _p, _p, _p, _p, _i, _p, _i, _i, _i, _p], _i),
    "fgm_cuda_gemm_q8c": ([_i, _i, _i, _p, _p, _p, _p, _p, _i, _i, _i, _p], _i),
    "fgm_cuda_gemm_q4g_warm": ([_i, _i, _i, _p, _p, _p, _p, _i, _p, _i, _i, _i,
                                _p, _sz, _p, _sz, _p], _i),
    "fgm_cuda_gemm_q8c_warm": ([_i, _i, _i, _p, _p, _p, _p, _p, _i, _i, _i,
                                _p, _sz, _p, _sz, _p], _i),
    "fgm_cuda_prep_rows": ([_p, _i, _p, _p, _p, _p, _i, _i, _i, _i, _i, _p], _i),
    "fgm_cuda_linear_q4g": ([_p, _i, _i, _i, _i, _i, _p, _p, _i, _p, _i, _i, _i, _p], _i),
    "fgm_cuda_linear_q8c": ([_p, _i, _i, _i, _i, _i, _p, _p, _p, _i, _i, _i, _p], _i),
    "fgm_cuda_q8c_prepare": ([_p, _i, _i, _p], _i),
    "fgm_cuda_gemm_q8c_rows": ([_i, _i, _i, _p, _i, _p, _p, _p, _p, _i, _i, _i, _p], _i),
    "fgm_cuda_q8c_release": ([_p], _i),
    "fgm_cuda_gemm_q8c_noalloc": ([_i, _i, _i, _p, _p, _p, _p, _p, _i, _i, _i, _p], _i),
    "fgm_cuda_worklist_create": ([_i, _p, _i, C.POINTER(_p)], _i),
    "fgm_cuda_worklist_run": ([_p, _p], _i),
    "fgm_cuda_worklist_destroy": ([_p], _i),
    "fgm_cuda_argmax_parts": ([_i], _i),
    "fgm_cuda_argmax_partials": ([_p, _i, _i, _i, _i, _p, _p, _p], _i),
    "fgm_cuda_argmax_merge": ([_p, _p, _i, _i, _p, _p], _i),
    "fgm_cuda_rmsnorm": ([_p, _p, _p, _i, _i, C.c_float, _p], _i),
    "fgm_cuda_gelu_mul": ([_p, _p, _p, _i, _i, _p], _i),
    "fgm_cuda_add": ([_p, _p, _sz, _p], _i),
    "fgm_cuda_mul": ([_p, _p, _sz, _p], _i),
    "fgm_cuda_scale": ([_p, C.c_float, _sz, _p], _i),
    "fgm_cuda_softcap": ([_p, _i, _i, C.c_float, _p], _i),
    "fgm_cuda_rope": ([_p, _i, _i, _i, _i, _p, _p, _p], _i),
    "fgm_cuda_rope_table": ([_p, _i, _i, _p], _i),
    "fgm_cuda_rope_cs": ([_p, _i, _i, _i, _i, _p, _p, _i, _p, _p], _i),
    "fgm_cuda_quant_act": ([_p, _i, _i, _p, _p, _p], _i),
    "fgm_cuda_store_v_t": ([_p, _sz, _p, _i, _i, _i, _i, _p], _i),
    "fgm_cuda_attend_q8": ([_p, _i, _p, _i, _p, _sz, _p, _sz, _p, _sz, _p, _sz, _i, _i, _i, _i,
                            _i, _i, _i, _p], _i),
    "fgm_cuda_norm_prep": ([_p, _p, _p, _p, _i, _i, C.c_float, _p, _p, _p], _i),
    "fgm_cuda_gelu_mul_prep": ([_p, _p, _i, _i, _i, _p, _p, _p, _p], _i),
    "fgm_cuda_qkv_post": ([_p, _i, _p, _p, _i, _i, _i, _i, _i, _p, _p, C.c_float, _p, _p, _i, _i,
                           _p, _sz, _p, _sz, _p, _sz, _p, _sz, _p], _i),
    "fgm_cuda_qkv_post_cs": ([_p, _i, _p, _p, _i, _i, _i, _i, _i, _p, _p, C.c_float, _p, _p, _i,
                              _p, _i, _i, _p, _sz, _p, _sz, _p, _sz, _p, _sz, _p], _i),
    "fgm_cuda_ipc_alloc": ([_sz, C.POINTER(_p)], _i),
    "fgm_cuda_ipc_free": ([_p], _i),
    "fgm_cuda_ipc_handle": ([_p, _p], _i),
    "fgm_cuda_ipc_open": ([_p, C.POINTER(_p)], _i),
    "fgm_cuda_ipc_close": ([_p], _i),
    "fgm_cuda_gemm_q4g_gather": ([_i, _i, _i, _p, _p, _p, _p, _i, _i, _i, _p, _p, _i, _i, _sz,
                                  _p], _i),
    "fgm_cuda_gemm_q4g_acc": ([_i, _i, _i, _p, _p, _i, _p, _i, _i, _p], _i),
    "fgm_cuda_gemm_q8c_acc": ([_i, _i, _i, _p, _p, _p, _i, _i, _p], _i),
}


class FgmCudaError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"fgm_cuda error {code}: {msg}")
        self.code = code


_lib = None


def lib():
    """The loaded library (loaded once; raises if it was never built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(
                f"{LIB_PATH} is missing: build it with `python -m fastgemma_b200.build`")
        L = C.CDLL(LIB_PATH)
        for name, (args, res) in SIGNATURES.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = res
        _lib = L
    return _lib


def check(rc: int) -> int:
    if rc < 0:
        raise FgmCudaError(rc, lib().fgm_cuda_last_error().decode())
    return rc


def call(name: str, *args) -> int:
    return check(getattr(lib(), name)(*args))
