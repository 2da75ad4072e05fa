"""The C-ABI library loads, exports every symbol include/fgm_cuda.h declares,
and rejects out-of-contract arguments on the host before touching a device."""
import ctypes as C
import os
import re

import numpy as np
import pytest

from fastgemma_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    names = set()
    for h in os.listdir(os.path.join(ROOT, "include")):
        if h.endswith(".h"):
            text = open(os.path.join(ROOT, "include", h)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            names |= set(re.findall(r"\b(fgm_\w+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    declared = header_symbols()
    assert declared, "no declarations parsed"
    missing = [s for s in declared if not hasattr(L, s)]
    assert not missing, missing
    # the Python binding covers the same set
    assert declared <= set(_lib.SIGNATURES), declared - set(_lib.SIGNATURES)


def test_last_error_empty_initially():
    assert isinstance(_lib.lib().fgm_cuda_last_error(), bytes)


def _q4g(M=8, N=64, K=128, group=64, ldc=None, n0=0, n1=4):
    a = np.zeros(16 * K, np.int8)
    s = np.ones(max(M, 1), np.float32)
    b = np.zeros(N * K // 2, np.uint8)
    bs = np.zeros((K // group if group > 0 else 1) * N, np.uint16)
    c = np.zeros(max(M, 1) * (ldc or N) + 64, np.float32)
    return _lib.lib().fgm_gemm_q4g_cuda(M, N, K, a.ctypes.data, s.ctypes.data, b.ctypes.data,
                                         bs.ctypes.data, group, c.ctypes.data, ldc or N, n0, n1)


@pytest.mark.parametrize("kw,frag", [
    (dict(K=100), "K=100"), (dict(K=0), "K=0"), (dict(N=24), "N=24"),
    (dict(group=32), "group=32"), (dict(group=96, K=128), "group=96"),
    (dict(n0=0, n1=3), "multiple of 4"), (dict(n0=4, n1=8), "outside"),
    (dict(ldc=32), "ldc=32"), (dict(M=-1), "M=-1")])
def test_contract_violations_rejected_on_host(kw, frag):
    rc = _q4g(**kw)
    assert rc == -1  # FGM_CUDA_EINVAL
    assert frag in _lib.lib().fgm_cuda_last_error().decode()


def test_empty_ranges_are_noops_without_device():
    assert _q4g(M=0) == 0
    assert _q4g(n0=4, n1=4) == 0


def test_group32_f32_scale_configs_rejected():
    # BASELINE config 0 names group-32 / f32 scales; the .fgm format (and both
    # reference kernels) admit only groups that are multiples of 64
    assert _q4g(group=32) == -1


def test_prep_contract():
    L = _lib.lib()
    x = np.zeros((4, 64), np.float32)
    qs = np.zeros(4, np.float32)
    pa = np.zeros(16 * 64, np.int8)
    # hsz not a power of two
    assert L.fgm_prep_rows_cuda(x.ctypes.data, 64, None, None, qs.ctypes.data, pa.ctypes.data,
                                4, 64, 48, 0, 4) == -1
    # r0 not tile aligned
    assert L.fgm_prep_rows_cuda(x.ctypes.data, 64, None, None, qs.ctypes.data, pa.ctypes.data,
                                4, 64, 0, 2, 4) == -1
    # lda < k
    assert L.fgm_prep_rows_cuda(x.ctypes.data, 32, None, None, qs.ctypes.data, pa.ctypes.data,
                                4, 64, 0, 0, 4) == -1


def test_availability_probe_reports_no_device_here():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a device is visible")
    assert _lib.lib().fgm_cuda_available() == 0


# ---- decode-step glue: argument contracts checked on the host, no device
_FAKE = 0x10000  # never dereferenced: every case below fails before any access


def _err():
    return _lib.lib().fgm_cuda_last_error().decode()


@pytest.mark.parametrize("kw,frag", [
    (dict(head_dim=96), "head_dim"), (dict(n_heads=6, kv_heads=4), "kv_heads"),
    (dict(start=0, end=200, ring=128), "ring"), (dict(end=0), "positions"),
    (dict(out_ld=100), "out_ld"), (dict(rows=2, kc_stride=64 * 256 - 1), "strides"),
    (dict(rows=2, vt_stride=64 * 256 - 4), "strides")])
def test_attention_contract(kw, frag):
    a = dict(out_ld=256, q_ld=256, kc_stride=64 * 256, ks_stride=64, vt_stride=64 * 256,
             vs_stride=64, rows=1, n_heads=1, kv_heads=1, head_dim=256, start=0, end=64, ring=0)
    a.update(kw)
    rc = _lib.lib().fgm_cuda_attend_q8(
        _FAKE, a["out_ld"], _FAKE, a["q_ld"], _FAKE, a["kc_stride"], _FAKE, a["ks_stride"], _FAKE,
        a["vt_stride"], _FAKE, a["vs_stride"], a["rows"], a["n_heads"], a["kv_heads"],
        a["head_dim"], a["start"], a["end"], a["ring"], None)
    assert rc == -1 and frag in _err(), _err()


def test_fused_glue_contracts():
    L = _lib.lib()
    # norm_prep: n a multiple of 64, at most 12288
    assert L.fgm_cuda_norm_prep(_FAKE, None, None, None, 2, 100, 1e-6, _FAKE, _FAKE, None) == -1
    assert "n=100" in _err()
    assert L.fgm_cuda_norm_prep(_FAKE, None, None, None, 2, 16384, 1e-6, _FAKE, _FAKE, None) == -1
    # gelu_mul_prep: rows of gate / up at least n apart
    assert L.fgm_cuda_gelu_mul_prep(_FAKE, _FAKE, 64, 2, 128, None, _FAKE, _FAKE, None) == -1
    assert "ld=64" in _err()
    # qkv_post: the ring must fit the cache, the row strides must hold it
    args = [_FAKE, 2048, _FAKE, _FAKE, 512, 2, 8, 2, 256, _FAKE, _FAKE, 1e-6, _FAKE, _FAKE]
    tail = [_FAKE, 1024 * 512, _FAKE, 1024, _FAKE, 1024 * 512, _FAKE, 1024, None]
    assert L.fgm_cuda_qkv_post(*args, 2048, 1024, *tail) == -1 and "ring" in _err()
    assert L.fgm_cuda_qkv_post(*args, 0, 2048, *tail) == -1 and "strides" in _err()
    bad_ld = list(args)
    bad_ld[1] = 1000
    assert L.fgm_cuda_qkv_post(*bad_ld, 0, 1024, *tail) == -1 and "q_ld=1000" in _err()
    # rows == 0 is a no-op that needs no device
    assert L.fgm_cuda_norm_prep(_FAKE, None, None, None, 0, 2048, 1e-6, _FAKE, _FAKE, None) == 0
