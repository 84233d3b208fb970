"""lnsb_soft_max_lns_noalloc: the allocation-free softmax entry point.

Some callers cannot call cudaMalloc at the point where they run the op:
a host framework whose own pool owns every device allocation, or a
latency-critical loop that may not take the allocator's implicit
synchronisation.  This entry point takes the
softmax scratch from a static device array compiled into the library instead
of a caller-provided work buffer.  The test calls it through the C ABI twice
in a row (different inputs, so the second call reuses the array the first
one wrote) and checks each result against the existing entry point
(lnsb_soft_max_lns with its own work buffer), bit for bit -- the tolerance
every parity test here uses.  It also checks that the size limit is refused,
including shapes whose element count would wrap a 64-bit integer, and that a
call after the first one leaves the device's free memory unchanged.

This file is collected last on purpose, and works both on its own in a fresh
process and after the rest of the suite.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _ne(shape):
    return (ctypes.c_int64 * 4)(*shape)


def _run_both(lib, fmt, src, shape, mask, mshape, scale):
    """(existing entry point with a work buffer, allocation-free entry point)"""
    dt = torch.int16 if fmt == 16 else torch.int32
    s = torch.from_numpy(src).cuda()
    m = torch.from_numpy(mask).cuda() if mask is not None else None
    n = src.size
    ref = torch.empty(n, dtype=dt, device="cuda")
    work = torch.empty(n, dtype=dt, device="cuda")
    out = torch.empty(n, dtype=dt, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    mp = ctypes.c_void_p(m.data_ptr()) if m is not None else None
    mne = _ne(mshape) if m is not None else None
    assert lib.lnsb_soft_max_lns(fmt, ctypes.c_void_p(s.data_ptr()), _ne(shape), mp, mne, scale,
                                 ctypes.c_void_p(ref.data_ptr()), ctypes.c_void_p(work.data_ptr()), 7, stream) == 0
    assert lib.lnsb_soft_max_lns_noalloc(fmt, ctypes.c_void_p(s.data_ptr()), _ne(shape), mp, mne, scale,
                                         ctypes.c_void_p(out.data_ptr()), 7, stream) == 0
    torch.cuda.synchronize()
    return ref.cpu().numpy(), out.cpu().numpy()


def test_noalloc_soft_max_matches_soft_max_lns():
    from lnsb200 import _lib
    lib = _lib.load("base")
    assert lib.lnsb_upload_tables(16) == 0          # one-time set-up (allocates the tables)
    assert lib.lnsb_upload_tables(32) == 0
    rng = np.random.default_rng(2024)

    # call 1: xlns16, 9 heads x 64 queries x 512 keys, causal mask, scale 1/8
    n, q, h = 512, 64, 9
    src = (rng.integers(0x3000, 0x5000, (h, q, n)) | (rng.integers(0, 2, (h, q, n)) << 15)).astype(np.uint16)
    mask = np.zeros((q, n), np.uint16)
    for i in range(q):
        mask[i, i + 1 + n - q:] = 0xFFFF                                  # xlns16 -inf
    ref1, got1 = _run_both(lib, 16, src.view(np.int16), (n, q, h, 1), mask.view(np.int16), (n, q, 1, 1), 0x3E80)
    assert np.array_equal(got1, ref1)

    # call 2, same array reused: a different shape, no mask
    src2 = (rng.integers(0x3800, 0x4800, (3, 40, 1100)) | (rng.integers(0, 2, (3, 40, 1100)) << 15)).astype(np.uint16)
    ref2, got2 = _run_both(lib, 16, src2.view(np.int16), (1100, 40, 3, 1), None, None, 0x4000)
    assert np.array_equal(got2, ref2)

    # xlns32 through the same array
    src3 = (rng.integers(0x3E000000, 0x42000000, (6, 300), dtype=np.int64) |
            (rng.integers(0, 2, (6, 300), dtype=np.int64) << 31)).astype(np.uint32)
    ref3, got3 = _run_both(lib, 32, src3.view(np.int32), (300, 6, 1, 1), None, None, 0x40000000)
    assert np.array_equal(got3, ref3)


def test_noalloc_refuses_beyond_its_scratch():
    from lnsb200 import _lib
    lib = _lib.load("base")
    assert lib.lnsb_upload_tables(16) == 0
    limit_elems = (8 << 20) // 2
    big = _ne((limit_elems + 1, 1, 1, 1))
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    dummy = torch.empty(16, dtype=torch.int16, device="cuda")
    st = lib.lnsb_soft_max_lns_noalloc(16, ctypes.c_void_p(dummy.data_ptr()), big, None, None, 0x4000,
                                       ctypes.c_void_p(dummy.data_ptr()), 7, stream)
    assert st == -4                                                          # LNSB_E_TOO_LARGE
    assert b"limit" in lib.lnsb_error_string(st)
    # element counts that wrap int64 (2^64 -> 0, 2^63 + small) are refused, not run
    for shape in ((1 << 32, 1 << 32, 1, 1), (1 << 31, 1 << 31, 4, 1), (3, 1 << 62, 2, 1)):
        st = lib.lnsb_soft_max_lns_noalloc(16, ctypes.c_void_p(dummy.data_ptr()), _ne(shape), None, None, 0x4000,
                                           ctypes.c_void_p(dummy.data_ptr()), 7, stream)
        assert st == -4, shape


def test_noalloc_allocates_nothing():
    """after the first call on a device (the one-time symbol lookup), a call
    leaves cudaMemGetInfo's free bytes exactly as they were"""
    from lnsb200 import _lib
    lib = _lib.load("base")
    assert lib.lnsb_upload_tables(16) == 0
    rng = np.random.default_rng(11)
    src = torch.from_numpy((rng.integers(0x3800, 0x4800, 64 * 700)).astype(np.uint16).view(np.int16)).cuda()
    out = torch.empty_like(src)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    call = lambda: lib.lnsb_soft_max_lns_noalloc(16, ctypes.c_void_p(src.data_ptr()), _ne((700, 64, 1, 1)), None,
                                                 None, 0x4000, ctypes.c_void_p(out.data_ptr()), 7, stream)
    assert call() == 0
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        assert call() == 0
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
