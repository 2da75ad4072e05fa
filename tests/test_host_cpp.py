"""The C++ host layer (fastgemma_b200/host: fgm_kernels / fgm_core over the C
ABI) through its own C++ test program, tests/cpp/host_layer_test.cpp."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "fastgemma_b200")
ORACLE = os.path.join(ROOT, "oracle")


@pytest.fixture(scope="module")
def host_test_bin(tmp_path_factory):
    from fastgemma_b200 import build as B
    B.build_host()
    exe = str(tmp_path_factory.mktemp("hostcpp") / "host_layer_test")
    cxx = shutil.which("g++") or "g++"
    cmd = [cxx, "-std=c++17", "-O2", "-Wall", "-I", os.path.join(ROOT, "include"),
           "-I", os.path.join(PKG, "host"), os.path.join(ROOT, "tests", "cpp", "host_layer_test.cpp"),
           "-o", exe, "-L", PKG, "-lfgm_host", "-lfgm_cuda", "-L", ORACLE, "-loracle",
           f"-Wl,-rpath,{PKG}:{ORACLE}"]
    subprocess.run(cmd, check=True)
    return exe


def _run(exe, mode):
    r = subprocess.run([exe, mode], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    return r.stdout


def test_host_layer_contracts_without_device(host_test_bin):
    import torch
    if torch.cuda.is_available():
        pytest.skip("the no-device checks need a machine without a GPU")
    out = _run(host_test_bin, "cpu")
    assert "0 failure(s)" in out


@pytest.mark.gpu
def test_host_layer_on_device(host_test_bin):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    out = _run(host_test_bin, "gpu")
    assert "0 failure(s)" in out and "backend: cuda" in out
