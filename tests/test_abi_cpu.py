"""The C ABI without a GPU: every library builds, loads and exports every
function include/lnsb200.h declares; identity, draw accounting and the Monte
state API (host-only calls) behave like the reference's
(lns-cuda-kernels.h:89-100, ggml-lns.h:13-24, ggml-lns-cuda.cpp:21-31)."""
import ctypes
import os
import re
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "lnsb200.h")
HEADERS = [HEADER, os.path.join(ROOT, "include", "lnsb200_graph.h")]
MODES = ("base", "monte", "monte_bylpvip", "lpvip", "sum32")


def declared():
    """every function the C headers declare (lnsb200.h, the host layer's lnsb200_graph.h)"""
    text = "".join(open(h).read() for h in HEADERS)
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(lnsb_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def libs():
    sys.path.insert(0, os.path.join(ROOT, "xlns-ggml-backend_b200"))
    import build
    build.build_all()
    from lnsb200 import _lib
    return {m: _lib.load(m) for m in MODES}


def test_header_declares_the_kernel_set_surface():
    names = declared()
    for fn in ("lnsb_format_name", "lnsb_value_size", "lnsb_sum_mode", "lnsb_monte_impl", "lnsb_mul_mat_draws",
               "lnsb_soft_max_draws", "lnsb_rms_norm_draws", "lnsb_upload_tables", "lnsb_to_lns",
               "lnsb_to_lns_transposed", "lnsb_mul_mat", "lnsb_soft_max", "lnsb_rms_norm"):
        assert fn in names


def test_every_declared_symbol_is_exported(libs):
    names = declared()
    from lnsb200 import _lib, graph
    bound = {n for n, _, _ in _lib.SIGNATURES} | {n for n, _, _ in graph._SIGS}
    for mode, lib in libs.items():
        for n in names:
            assert hasattr(lib, n), "%s missing from liblnsb200_%s.so" % (n, mode)
    missing = [n for n in names if n not in bound]
    assert not missing, "header functions without a binding: %s" % missing


def test_identity(libs):
    for mode, lib in libs.items():
        assert lib.lnsb_format_name(16) == b"xlns16" and lib.lnsb_format_name(32) == b"xlns32"
        assert lib.lnsb_format_name(8) is None
        assert lib.lnsb_value_size(16) == 2 and lib.lnsb_value_size(32) == 4
        want = b"monte" if mode.startswith("monte") else mode.encode()
        assert lib.lnsb_sum_mode(16) == want
        assert lib.lnsb_sum_mode(32) is None
        impl = {"monte": b"pure16", "monte_bylpvip": b"bylpvip"}.get(mode)
        assert lib.lnsb_monte_impl(16) == impl
        desc = lib.lnsb_description(16).decode()
        assert "sum=%s" % want.decode() in desc
        if impl:
            assert "monte=%s" % impl.decode() in desc
        assert b"xlns32" in lib.lnsb_description(32)


def test_draws(libs, orc):
    from lnsb200 import MulMatArgs
    for mode, lib in libs.items():
        for K, M, N, ne12, ne13 in [(1536, 576, 8, 1, 1), (1, 3, 3, 1, 1), (0, 3, 3, 1, 1), (17, 5, 6, 4, 2)]:
            a = MulMatArgs(None, None, None, K, M, N, 1, 1, ne12, ne13, 7)
            assert lib.lnsb_mul_mat_draws(16, ctypes.byref(a)) == orc.lib().orc_mul_mat_draws(orc.MODE[mode], K, M, N, ne12, ne13)
            assert lib.lnsb_mul_mat_draws(32, ctypes.byref(a)) == 0
        assert lib.lnsb_soft_max_draws(16, 512, 4608) == orc.lib().orc_soft_max_draws(orc.MODE[mode], 512, 4608)
        assert lib.lnsb_soft_max_draws(16, 0, 4) == 0
        assert lib.lnsb_rms_norm_draws(16, 576, 512) == orc.lib().orc_rms_norm_draws(orc.MODE[mode], 576, 512)


def test_monte_state(libs, orc):
    for mode, lib in libs.items():
        s = ctypes.c_uint16()
        if not mode.startswith("monte"):
            assert lib.lnsb_monte_get_state(ctypes.byref(s)) == -3
            assert lib.lnsb_monte_set_state(5) == -3
            continue
        assert lib.lnsb_monte_set_state(7) == 0
        assert lib.lnsb_monte_get_state(ctypes.byref(s)) == 0 and s.value == 7
        assert lib.lnsb_monte_set_state(0) == -1             # 0 is absorbing: rejected
        start = ctypes.c_uint16()
        assert lib.lnsb_monte_reserve(1, ctypes.byref(start)) == 0 and start.value == 7
        assert lib.lnsb_monte_get_state(ctypes.byref(s)) == 0 and s.value == 0xB403   # one LFSR step
        assert lib.lnsb_monte_reserve(10 ** 12 + 3, ctypes.byref(start)) == 0 and start.value == 0xB403
        assert lib.lnsb_monte_get_state(ctypes.byref(s)) == 0
        assert s.value == orc.lfsr_jump(0xB403, 10 ** 12 + 3)
        assert lib.lnsb_monte_set_state(7) == 0


def test_error_strings(libs):
    lib = libs["base"]
    assert lib.lnsb_error_string(0) == b"success"
    assert b"upload_tables" in lib.lnsb_error_string(-2)
    assert lib.lnsb_error_string(-1) == b"invalid argument"
