"""lnsb_mul_mat_xf32 -- the MUL_MAT op over F32 activations (the reference's
compute_mul_mat, lns-backend/cuda/lns-cuda-ops.cpp:57-75: to_lns of src1, then
kernel_set::mul_mat) -- against the oracle, bit for bit.

The weight-resident latency kernel converts the activations while it stages
them (16-byte loads where K is a multiple of 8 and x is 16-byte aligned, one
value per load otherwise); every other kernel reads codes converted into
x_work first.  The shapes reach both, and both staging forms of the first.
"""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

MODES = ("base", "monte", "monte_bylpvip", "lpvip", "sum32")
NT = os.cpu_count() or 1


@pytest.fixture(scope="module", params=MODES)
def ks16(request):
    from lnsb200 import KernelSet
    k = KernelSet(16, request.param)
    k.upload_tables()
    return k


@pytest.fixture(scope="module")
def ks32():
    from lnsb200 import KernelSet
    k = KernelSet(32, "base")
    k.upload_tables()
    return k


def activations(rng, shape):
    """N(0, 1) floats with zeros, negative zeros, tiny and huge values mixed in"""
    x = rng.normal(0.0, 1.0, shape).astype(np.float32)
    flat = x.reshape(-1)
    pick = rng.choice(flat.size, size=max(1, flat.size // 50), replace=False)
    specials = np.array([0.0, -0.0, 1e-30, -3e-38, 7e30, -1.0, 1.0, 2.0 ** -20], np.float32)
    flat[pick] = specials[rng.integers(0, specials.size, pick.size)]
    return x


def run_xf32(ks, w_rows, xf, slices=(1, 1, 1, 1), seed=7, misalign=False):
    """w_rows codes [ne03][ne02][M][K], xf F32 [ne13][ne12][N][K] -> F32 result"""
    M, K = w_rows.shape[-2], w_rows.shape[-1]
    N = xf.shape[-2]
    it, dt = (np.int16, torch.int16) if ks.fmt == 16 else (np.int32, torch.int32)
    wd = torch.from_numpy(np.ascontiguousarray(np.swapaxes(w_rows, -1, -2)).view(it)).cuda()
    flat = torch.from_numpy(np.ascontiguousarray(xf).reshape(-1))
    if misalign:                                     # 4 bytes past a 16-byte boundary
        buf = torch.empty(flat.numel() + 1, dtype=torch.float32, device="cuda")
        buf[1:].copy_(flat)
        xd = buf[1:]
    else:
        xd = flat.cuda()
    work = torch.full((max(1, flat.numel()),), -1, dtype=dt, device="cuda")
    out = torch.empty(slices[2] * slices[3] * N * M, dtype=torch.float32, device="cuda")
    ks.mul_mat_xf32(wd, xd, work, out, K, M, N, slices, seed)
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("K,M,N,misalign", [
    (1536, 576, 8, False),   # the latency kernel, 16-byte staging
    (1536, 576, 8, True),    # the same with x off the 16-byte boundary: one value per load
    (7, 40, 5, False),       # K not a multiple of 8
    (4096, 64, 2, False),    # the longest K the latency kernel takes
    (1, 64, 8, False),       # K = 1
    (200, 37, 1, False),     # a decode row, odd M
    (576, 1536, 512, False), # configs[1]: the tiled kernel over x_work
    (40, 2048, 640, False),  # the throughput kernels over x_work
])
def test_mul_mat16_xf32(orc, ks16, K, M, N, misalign):
    rng = np.random.default_rng(K * 131 + M * 7 + N)
    w = orc.from_f32_16(rng.normal(0.0, 0.02, (M, K)).astype(np.float32))
    xf = activations(rng, (N, K))
    want = orc.to_f32_16(orc.mul_mat16(ks16.mode, w, orc.from_f32_16(xf), seed=7, nthreads=NT)).ravel()
    got = run_xf32(ks16, w, xf, seed=7, misalign=misalign)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), \
        "first mismatch at %d" % np.flatnonzero(got.view(np.uint32) != want.view(np.uint32))[0]


def test_mul_mat16_xf32_broadcast_slices(orc, ks16):
    """activation slice (i12, i13) over weight slice (i12 / 2, i13 / 2)"""
    rng = np.random.default_rng(6)
    slices = (2, 1, 4, 2)
    M, K, N = 32, 72, 9
    w = orc.from_f32_16(rng.normal(0.0, 0.5, (1, 2, M, K)).astype(np.float32))
    xf = activations(rng, (2, 4, N, K))
    want = orc.to_f32_16(orc.mul_mat16(ks16.mode, w, orc.from_f32_16(xf), slices=slices, seed=3, nthreads=NT)).ravel()
    got = run_xf32(ks16, w, xf, slices=slices, seed=3)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("K,M,N", [(576, 96, 9), (7, 40, 5), (1536, 576, 8)])
def test_mul_mat32_xf32(orc, ks32, K, M, N):
    rng = np.random.default_rng(K + 3 * M + N)
    w = orc.from_f32_32(rng.normal(0.0, 0.02, (M, K)).astype(np.float32))
    xf = activations(rng, (N, K))
    want = orc.to_f32_32(orc.mul_mat32(w, orc.from_f32_32(xf), nthreads=NT)).ravel()
    got = run_xf32(ks32, w, xf)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_mul_mat_xf32_requires_x_work(ks16):
    import ctypes
    import lnsb200
    w = torch.zeros(8 * 4, dtype=torch.int16, device="cuda")
    x = torch.zeros(2 * 8, dtype=torch.float32, device="cuda")
    out = torch.zeros(2 * 4, dtype=torch.float32, device="cuda")
    a = lnsb200.MulMatArgs(w.data_ptr(), x.data_ptr(), out.data_ptr(), 8, 4, 2, 1, 1, 1, 1, 7)
    st = ks16.lib.lnsb_mul_mat_xf32(16, ctypes.byref(a), None, None)
    assert st == -1                                  # LNSB_E_INVALID
    a0 = lnsb200.MulMatArgs(w.data_ptr(), x.data_ptr(), out.data_ptr(), 0, 4, 2, 1, 1, 1, 1, 7)
    assert ks16.lib.lnsb_mul_mat_xf32(16, ctypes.byref(a0), None, None) == 0   # K = 0 needs none
    torch.cuda.synchronize()
    assert bool((out == 0).all())                    # the empty sum: zero
