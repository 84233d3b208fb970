"""Builds the B200 LNS libraries in-tree: lib/liblnsb200_<mode>.so, one per
xlns16 summation mode, exactly as the reference builds one tree per
GGML_LNS16_SUM mode (lns-backend/common/lns-common.cmake:24-46).  Every
library also carries the xlns32 (LNSCUDA32) kernels.

    python xlns-ggml-backend_b200/build.py            # all modes
    python xlns-ggml-backend_b200/build.py base sum32 # some
"""
import concurrent.futures
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "lib")

# mode name -> LNSB_SUM_MODE value (csrc/lnsb_arith.cuh)
MODES = {"base": 0, "monte": 1, "monte_bylpvip": 2, "lpvip": 3, "sum32": 4}

SOURCES = ["lnsb_kernels.cu", "lnsb_tables.cpp", "lnsb_graph.cpp"]
HEADERS = ["lnsb_arith.cuh", "lnsb_tables.h", os.path.join(ROOT, "include", "lnsb200.h"),
           os.path.join(ROOT, "include", "lnsb200_graph.h")]


def nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.isabs(cand) and os.path.exists(cand) or not os.path.isabs(cand)):
            return cand
    return "nvcc"


def lib_path(mode):
    return os.path.join(LIB, "liblnsb200_%s.so" % mode)


def _stale(out):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    deps = [os.path.join(CSRC, s) for s in SOURCES] + [h if os.path.isabs(h) else os.path.join(CSRC, h) for h in HEADERS]
    return any(os.path.getmtime(d) > t for d in deps)


def build_mode(mode, force=False, verbose=False):
    out = lib_path(mode)
    if not force and not _stale(out):
        return out
    os.makedirs(LIB, exist_ok=True)
    cmd = [
        nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
        "-Xcompiler", "-fPIC,-ffp-contract=off", "-shared",
        "-DLNSB_SUM_MODE=%d" % MODES[mode],
        "-I", os.path.join(ROOT, "include"),
        "-o", out + ".tmp",
    ] + [os.path.join(CSRC, s) for s in SOURCES]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed for mode %s:\n%s\n%s" % (mode, " ".join(cmd), r.stderr))
    os.replace(out + ".tmp", out)
    return out


def build_all(modes=None, force=False):
    modes = list(modes or MODES)
    with concurrent.futures.ThreadPoolExecutor(max_workers=len(modes)) as ex:
        return list(ex.map(lambda m: build_mode(m, force), modes))


if __name__ == "__main__":
    names = [a for a in sys.argv[1:] if not a.startswith("-")]
    for p in build_all(names or None, force="--force" in sys.argv):
        print(p)
