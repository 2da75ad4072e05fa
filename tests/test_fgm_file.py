""".fgm model files: the Python reader (fastgemma_b200/fgm_file.py) and the
C++ loader (fastgemma_b200/host/fgm_model.hpp) against a fixture written by
the reference's own writer (tests/golden/make_fgm_fixture.py), against each
other, and on the device (registered weights, Gemm::run vs the oracle)."""
import importlib.util
import os
import shutil
import struct
import subprocess

import numpy as np
import pytest

from fastgemma_b200 import fgm_format as F
from fastgemma_b200.fgm_file import FgmError, FgmFile

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "fastgemma_b200")
ORACLE = os.path.join(ROOT, "oracle")
TINY = os.path.join(ROOT, "tests", "golden", "tiny.fgm")


def _fixture_module():
    spec = importlib.util.spec_from_file_location(
        "make_fgm_fixture", os.path.join(ROOT, "tests", "golden", "make_fgm_fixture.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="module")
def model_test_bin(tmp_path_factory):
    from fastgemma_b200 import build as B
    B.build_host()
    exe = str(tmp_path_factory.mktemp("fgmcpp") / "fgm_model_test")
    cxx = shutil.which("g++") or "g++"
    subprocess.run([cxx, "-std=c++17", "-O2", "-Wall", "-I", os.path.join(ROOT, "include"),
                    "-I", os.path.join(PKG, "host"), os.path.join(ROOT, "tests", "cpp",
                                                                  "fgm_model_test.cpp"),
                    "-o", exe, "-L", PKG, "-lfgm_host", "-lfgm_cuda", "-L", ORACLE, "-loracle",
                    f"-Wl,-rpath,{PKG}:{ORACLE}"], check=True)
    return exe


def _run(exe, *args):
    r = subprocess.run([exe, *args], capture_output=True, text=True, timeout=300)
    return r.returncode, r.stdout + r.stderr


def test_reader_returns_what_the_reference_writer_stored():
    """Every linear of the fixture: blob == this repo's packing of the same
    seeded weights (the .fgm tile layouts), scales, meta, twins, config."""
    mk = _fixture_module()
    f = FgmFile(TINY)
    assert f.arch == "gemma3n" and f.config["hidden_size"] == 256
    assert f.meta["generator"] == "tests/golden/make_fgm_fixture.py"
    for name, bits, n, k, group, had, twin, seed in mk.LINEARS:
        lin = f.linear(name)
        assert (lin["bits"], lin["n"], lin["k"], lin["hadamard"]) == (bits, n, k, had)
        q, s = mk.weights(bits, n, k, group, seed)
        if bits == 4:
            assert lin["group"] == group
            assert np.array_equal(np.asarray(lin["q"]), F.pack_q4g(q))
            assert np.array_equal(np.asarray(lin["scale"]), s.view(np.uint16).reshape(-1))
        else:
            assert lin["group"] == 0
            assert np.array_equal(np.asarray(lin["q"]), F.pack_b_tiles(q).view(np.int8))
            assert np.array_equal(np.asarray(lin["scale"]), s)
        lo, hi = f.dual(name)
        assert (hi is not None) == twin
        if twin:
            q8, s8 = mk.weights(8, n, k, 0, seed + 100)
            assert hi["bits"] == 8 and np.array_equal(np.asarray(hi["q"]),
                                                      F.pack_b_tiles(q8).view(np.int8))
            assert np.array_equal(np.asarray(hi["scale"]), s8)
    for e in f.tensors.values():
        assert e["offset"] % 64 == 0  # blobs are 64-byte aligned
    assert f.total_bytes() == sum(e["nbytes"] for e in f.tensors.values())
    with pytest.raises(FgmError, match="missing tensor"):
        f.linear("no.such.tensor")
    with pytest.raises(FgmError, match="non-linear dtype"):
        f.linear("layers.0.input_layernorm.weight")


def _fnv1a(b: bytes) -> int:
    h = 1469598103934665603
    for x in b:
        h = ((h ^ x) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h


def test_cpp_loader_agrees_with_python_reader(model_test_bin):
    rc, out = _run(model_test_bin, "summary", TINY)
    assert rc == 0, out
    f = FgmFile(TINY)
    want = []
    for name in sorted(f.tensors):
        e = f.tensors[name]
        want.append(f"T {name} {e['dtype']} {','.join(map(str, e['shape']))} {e['offset']} "
                    f"{e['nbytes']} {_fnv1a(bytes(f.raw(name))):016x}")
        if e["dtype"] in ("q4g", "q8c"):
            lin = f.linear(name)
            want.append(f"L {name} {lin['bits']} {lin['n']} {lin['k']} {lin['group']} "
                        f"{lin['hadamard']} {lin['q'].size} {lin['scale'].size}")
            want.append(f"D {name} {int(f.dual(name)[1] is not None)}")
    want += [f"TOTAL {f.total_bytes()}", "CFG hidden_size 256", "CFG quant.ffn 4",
             "META generator tests/golden/make_fgm_fixture.py"]
    assert out.splitlines() == want


def _write_malformed(d):
    good = open(TINY, "rb").read()
    (hlen,) = struct.unpack("<I", good[8:12])
    files = {
        "good.fgm": good,
        "bad_magic.fgm": b"FASTGEM2" + good[8:],
        "short.fgm": good[:10],
        "header_past_end.fgm": good[:8] + struct.pack("<I", len(good)) + good[12:],
        "bad_json.fgm": good[:12] + b"{" * 3 + good[15:],
    }
    # a tensor entry pointing past the end of the file (same header length)
    hdr = good[12:12 + hlen].decode()
    bigger = hdr.replace('"nbytes":1024', '"nbytes":9999999', 1)
    assert bigger != hdr
    files["tensor_past_end.fgm"] = (good[:8] + struct.pack("<I", len(bigger)) + bigger.encode()
                                    + good[12 + hlen + (len(bigger) - hlen):])
    for name, data in files.items():
        with open(os.path.join(d, name), "wb") as fh:
            fh.write(data)
    return files


def test_malformed_files_are_rejected(tmp_path, model_test_bin):
    files = _write_malformed(str(tmp_path))
    for name in files:
        if name == "good.fgm":
            FgmFile(str(tmp_path / name))
            continue
        with pytest.raises(FgmError):
            FgmFile(str(tmp_path / name))
    rc, out = _run(model_test_bin, "errors", str(tmp_path))
    assert rc == 0 and "0 failure(s)" in out, out


@pytest.mark.gpu
def test_cpp_loader_on_device(model_test_bin):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    rc, out = _run(model_test_bin, "gpu", TINY)
    assert rc == 0 and "0 failure(s)" in out and "backend: cuda" in out, out


@pytest.mark.gpu
def test_python_reader_registers_and_runs_on_device(orc):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from fastgemma_b200 import _lib
    import fastgemma_b200.device  # noqa: F401
    import fastgemma_b200 as fg
    L = _lib.lib()
    f = FgmFile(TINY)
    before = L.fgm_cuda_registry_bytes()
    reg = f.register_linears()
    assert reg > 0 and L.fgm_cuda_registry_bytes() == before + reg
    lin = f.linear("layers.0.mlp.gate_proj")
    M, K, N = 8, lin["k"], lin["n"]
    x = F.synth_x(M, K, 3)
    c = np.zeros((M, N), np.float32)
    _lib.call("fgm_linear_q4g_cuda", x.ctypes.data, K, lin["hadamard"], M, N, K,
              lin["q"].ctypes.data, lin["scale"].ctypes.data, lin["group"], c.ctypes.data, N)
    _, _, qs, pa = orc.prep_rows(x, M, K, lin["hadamard"])
    want = orc.gemm_q4g(M, N, K, pa, qs, np.asarray(lin["q"]), np.asarray(lin["scale"]).view(
        np.float16), lin["group"])
    assert np.array_equal(c.view(np.uint32), want.view(np.uint32))
    f.unregister_linears()
    assert L.fgm_cuda_registry_bytes() == before
    del fg
