"""The xlns32 additions of the per-element kernels (the norm block's residual
add, the elementwise ops, the soft_max mask, the sigmoid) use the flat
image's branch-free adder (add32f); the chains of the other kernels that read
the separate tables use the branching one.  Both must give the same bits:
tests/cpp/flat_adder_check.cu restates the branching adder on the host tables
and compares the two over every small difference, the tables' end and random
pairs (host-only build with nvcc; no GPU)."""
import os
import shutil
import subprocess

import pytest

from conftest import ROOT

CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def test_flat_adder_equals_table_adder(tmp_path):
    nvcc = shutil.which("nvcc") or os.path.join(CUDA, "bin", "nvcc")
    if not os.path.exists(nvcc):
        pytest.skip("nvcc not available")
    csrc = os.path.join(ROOT, "xlns-ggml-backend_b200", "csrc")
    exe = str(tmp_path / "flat_adder_check")
    cmd = [nvcc, "-O2", "-std=c++17", "-DLNSB_SUM_MODE=0", "-I", csrc, "-I", os.path.join(ROOT, "include"),
           os.path.join(ROOT, "tests", "cpp", "flat_adder_check.cu"), os.path.join(csrc, "lnsb_tables.cpp"), "-o", exe]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]
    r = subprocess.run([exe, "20000000"], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:]
    n, bad = r.stdout.split()[0], r.stdout.split()[2]
    assert bad == "0" and int(n) > 50000000, r.stdout
