"""The C++ host interface (include/lnsb200_kernel_set.hpp, the reference's
kernel_set over the C ABI) compiled and linked against every mode's library,
and on a GPU its parity program run against the CPU oracle
(tests/cpp/kernel_set_parity.cpp)."""
import os
import shutil
import subprocess

import pytest

from conftest import ROOT

MODES = ("base", "monte", "monte_bylpvip", "lpvip", "sum32")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
LIB = os.path.join(ROOT, "xlns-ggml-backend_b200", "lib")
ORACLE = os.path.join(ROOT, "oracle", "_build")


def _build(mode, outdir):
    cxx = shutil.which("g++") or "g++"
    exe = os.path.join(outdir, "kernel_set_parity_" + mode)
    cmd = [cxx, "-O2", "-std=c++17", "-Wall", "-I", os.path.join(ROOT, "include"), "-I", os.path.join(ROOT, "oracle"),
           "-I", os.path.join(CUDA, "include"), os.path.join(ROOT, "tests", "cpp", "kernel_set_parity.cpp"),
           "-L", LIB, "-llnsb200_" + mode, "-L", ORACLE, "-llns_oracle", "-L", os.path.join(CUDA, "lib64"), "-lcudart",
           "-Wl,-rpath," + LIB, "-Wl,-rpath," + ORACLE, "-Wl,-rpath," + os.path.join(CUDA, "lib64"), "-o", exe]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]
    return exe


@pytest.fixture(scope="module")
def built(tmp_path_factory, orc):
    import build                                   # xlns-ggml-backend_b200/build.py
    build.build_all()                              # no-op when the libraries are current
    d = tmp_path_factory.mktemp("cpp")
    return {m: _build(m, str(d)) for m in MODES}


def test_cpp_interface_builds_for_every_mode(built):
    for m, exe in built.items():
        assert os.path.isfile(exe), m


@pytest.mark.gpu
@pytest.mark.parametrize("mode", MODES)
def test_cpp_kernel_set_parity(built, mode):
    r = subprocess.run([built[mode]], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
    assert "0 failed" in r.stdout
