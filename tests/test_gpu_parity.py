"""GPU == oracle, bit for bit, through the C ABI (include/lnsb200.h).

Mirrors the reference's parity harness (lns-backend/tests/test-lns-cuda-parity.cpp:
255-366): mul_mat over long K, K=1, N=1, ragged tiles and broadcast slices;
softmax with padded masks and long rows; rms_norm; the F32 boundary
conversions; every summation-mode build and the xlns32 format.  Results are
compared as integer codes (memcmp semantics, test-lns-cuda-parity.cpp:158-171).
"""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

MODES = ("base", "monte", "monte_bylpvip", "lpvip", "sum32")
NT = os.cpu_count() or 1


def dev16(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.uint16).view(np.int16)).cuda()


def dev32(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.uint32).view(np.int32)).cuda()


def host16(t):
    torch.cuda.synchronize()
    return t.cpu().numpy().view(np.uint16)


def host32(t):
    torch.cuda.synchronize()
    return t.cpu().numpy().view(np.uint32)


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


def codes16(orc, rng, shape, sigma):
    return orc.from_f32_16(rng.normal(0.0, sigma, shape).astype(np.float32))


def run_mm16(ks, w_rows, x, slices=(1, 1, 1, 1), seed=7, f32=False):
    """w_rows [ne03][ne02][M][K], x [ne13][ne12][N][K] -> GPU result (codes or f32)."""
    M, K = w_rows.shape[-2], w_rows.shape[-1]
    N = x.shape[-2]
    w_km = np.ascontiguousarray(np.swapaxes(w_rows, -1, -2))     # k-major [..][K][M]
    wd, xd = dev16(w_km), dev16(x)
    nout = slices[2] * slices[3] * N * M
    if f32:
        out = torch.empty(nout, dtype=torch.float32, device="cuda")
        ks.mul_mat(wd, xd, out, K, M, N, slices, seed)
        torch.cuda.synchronize()
        return out.cpu().numpy()
    out = torch.empty(nout, dtype=torch.int16, device="cuda")
    ks.mul_mat_lns(wd, xd, out, K, M, N, slices, seed)
    return host16(out)


# ----------------------------------------------------------------- mul_mat

@pytest.mark.parametrize("K,M,N", [
    (1536, 576, 8),      # BASELINE configs[0] shape
    (576, 1536, 64),     # configs[1] shape, 64 of its 512 tokens
    (576, 1536, 512),    # configs[1] in full (the tiled throughput kernel)
    (96, 1024, 640),     # tiled kernel, K tail in the last chunk
    (1, 64, 8),          # K=1: no addition at all
    (2, 32, 3),
    (7, 40, 5),          # K not a multiple of 8, M not a multiple of 32
    (65, 96, 65),        # one full K chunk + 1; ragged token tile
    (200, 37, 1),        # N=1 (decode), odd M
    (4096, 64, 2),       # long K
    (40, 2048, 640),     # enough units for two tokens per lane (sum32 flat-add kernel)
])
def test_mul_mat16(orc, ks16, K, M, N):
    rng = np.random.default_rng(K * 7919 + M * 31 + N)
    w = codes16(orc, rng, (M, K), 0.02)
    x = codes16(orc, rng, (N, K), 1.0)
    want = orc.mul_mat16(ks16.mode, w, x, seed=7, nthreads=NT).ravel()
    got = run_mm16(ks16, w, x, seed=7)
    assert np.array_equal(got, want), "first mismatch at %d" % np.flatnonzero(got != want)[0]


def test_mul_mat16_f32_out(orc, ks16):
    rng = np.random.default_rng(11)
    w = codes16(orc, rng, (64, 300), 0.02)
    x = codes16(orc, rng, (5, 300), 1.0)
    want = orc.to_f32_16(orc.mul_mat16(ks16.mode, w, x, seed=123, nthreads=NT)).ravel()
    got = run_mm16(ks16, w, x, seed=123, f32=True)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_mul_mat16_broadcast_slices(orc, ks16):
    """GQA-style broadcast: activation slice (i12, i13) uses weight slice
    (i12 / (ne12/ne02), i13 / (ne13/ne03)) (lns-cuda-kernels.h:45-50)."""
    rng = np.random.default_rng(5)
    ne02, ne03, ne12, ne13 = 2, 1, 4, 2
    M, K, N = 32, 72, 9
    w = codes16(orc, rng, (ne03, ne02, M, K), 0.5)
    x = codes16(orc, rng, (ne13, ne12, N, K), 1.0)
    want = orc.mul_mat16(ks16.mode, w, x, slices=(ne02, ne03, ne12, ne13), seed=99, nthreads=NT).ravel()
    got = run_mm16(ks16, w, x, slices=(ne02, ne03, ne12, ne13), seed=99)
    assert np.array_equal(got, want)


def test_mul_mat16_special_codes(orc, ks16):
    """zeros, signed zeros, saturated codes, exact cancellation pairs"""
    rng = np.random.default_rng(3)
    M, K, N = 64, 96, 16
    w = codes16(orc, rng, (M, K), 1.0)
    x = codes16(orc, rng, (N, K), 1.0)
    specials = np.array([0x0000, 0x8000, 0x7FFF, 0xFFFF, 0x4000, 0xC000, 0x0001, 0x3FFF], np.uint16)
    w.ravel()[rng.integers(0, w.size, 400)] = rng.choice(specials, 400)
    x.ravel()[rng.integers(0, x.size, 200)] = rng.choice(specials, 200)
    x[3] = x[2] ^ 0x8000          # token 3 = -token 2: cancelling products
    w[5, :] = 0x4000
    want = orc.mul_mat16(ks16.mode, w, x, seed=0xB403, nthreads=NT).ravel()
    got = run_mm16(ks16, w, x, seed=0xB403)
    assert np.array_equal(got, want)


def test_mul_mat16_tiled_slices_ragged(orc, ks16):
    """Enough outputs for the tiled kernels (base: the four-group kernel) with
    two activation slices over one weight slice, M not a multiple of the
    64-row tile and K not a multiple of 8 (the unaligned staging path),
    scattered special codes, codes and F32 out."""
    rng = np.random.default_rng(29)
    ne02, ne03, ne12, ne13 = 1, 1, 2, 1
    M, K, N = 1000, 70, 600
    w = codes16(orc, rng, (ne03, ne02, M, K), 0.02)
    x = codes16(orc, rng, (ne13, ne12, N, K), 1.0)
    specials = np.array([0x0000, 0x8000, 0x7FFF, 0xFFFF, 0x4000, 0xC000], np.uint16)
    w.ravel()[rng.integers(0, w.size, 50)] = rng.choice(specials, 50)
    x.ravel()[rng.integers(0, x.size, 50)] = rng.choice(specials, 50)
    sl = (ne02, ne03, ne12, ne13)
    want = orc.mul_mat16(ks16.mode, w, x, slices=sl, seed=41, nthreads=NT).ravel()
    assert np.array_equal(run_mm16(ks16, w, x, slices=sl, seed=41), want)
    got = run_mm16(ks16, w, x, slices=sl, seed=41, f32=True)
    assert np.array_equal(got.view(np.uint32), orc.to_f32_16(want).view(np.uint32))


@pytest.mark.parametrize("where", ["early", "late", "none"])
@pytest.mark.parametrize("M,K,N", [(128, 300, 40), (1024, 100, 640)])
def test_mul_mat16_range_fallback(orc, ks16, where, M, K, N):
    """A zero operand (or a huge one) part-way along K: the base kernels'
    key-form fast path must hand the chains over to packed codes at that
    point and still match bit for bit (small shape: latency kernel; large:
    tiled kernel)."""
    rng = np.random.default_rng(17)
    w = codes16(orc, rng, (M, K), 0.02)
    x = codes16(orc, rng, (N, K), 1.0)
    if where == "early":
        x[3, 5] = 0x0000            # exact zero in the first chunk
    elif where == "late":
        w[7, K - 50] = 0x0000       # zero in a later chunk
        x[11, K - 49] = 0x7FF0      # and a huge activation
    want = orc.mul_mat16(ks16.mode, w, x, seed=3, nthreads=NT).ravel()
    got = run_mm16(ks16, w, x, seed=3)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("K,M,N", [(1536, 96, 8), (700, 64, 3)])
def test_mul_mat16_zeros_scattered(orc, ks16, K, M, N):
    """Zero weights and activations scattered along K (pruned weights, padded
    activations): chains drop to packed codes around each zero and return to
    the key form where the operands allow, several times per chain."""
    rng = np.random.default_rng(K + N)
    w = codes16(orc, rng, (M, K), 0.02)
    x = codes16(orc, rng, (N, K), 1.0)
    for k in (3, 300, 555, 1000, 1290):
        if k < K:
            w[rng.integers(0, M, 4), k] = 0x0000
    for k in (40, 520, 1400):
        if k < K:
            x[rng.integers(0, N), k] = rng.choice(np.array([0x0000, 0x8000], np.uint16))
    want = orc.mul_mat16(ks16.mode, w, x, seed=11, nthreads=NT).ravel()
    got = run_mm16(ks16, w, x, seed=11)
    assert np.array_equal(got, want)


def test_draw_accounting(ks16, orc):
    for args in [(1536, 576, 8, 1, 1), (1, 4, 4, 1, 1), (0, 4, 4, 1, 1), (10, 3, 5, 4, 2)]:
        K, M, N, ne12, ne13 = args
        assert ks16.mul_mat_draws(K, M, N, 1, 1, ne12, ne13) == orc.lib().orc_mul_mat_draws(
            orc.MODE[ks16.mode], K, M, N, ne12, ne13)
    assert ks16.soft_max_draws(512, 4608) == orc.lib().orc_soft_max_draws(orc.MODE[ks16.mode], 512, 4608)
    assert ks16.rms_norm_draws(576, 512) == orc.lib().orc_rms_norm_draws(orc.MODE[ks16.mode], 576, 512)


# ----------------------------------------------------------------- soft_max

def causal_mask16(orc, nq, nk, pad_rows=0):
    m = np.zeros((nq + pad_rows, nk), np.float32)
    for q in range(nq + pad_rows):
        m[q, q + 1:] = -np.inf
    return orc.mask16(m)


@pytest.mark.parametrize("shape,masked,pad,scale", [
    ((64, 64, 9, 1), True, 0, 1.0),         # configs[1] softmax: causal, 9 heads (64 of 512 queries)
    ((512, 4, 1, 1), False, 0, 0.125),
    ((1100, 3, 2, 1), False, 0, 1.0),       # long rows (test-lns-cuda-parity.cpp)
    ((48, 10, 3, 2), True, 6, 0.5),         # padded mask rows, broadcast over dims 2/3
    ((1, 5, 1, 1), True, 0, 1.0),           # n = 1
])
def test_soft_max16(orc, ks16, shape, masked, pad, scale):
    n, r1, r2, r3 = shape
    rng = np.random.default_rng(n + r1)
    src = codes16(orc, rng, (r3, r2, r1, n), 3.0)
    src.ravel()[rng.integers(0, src.size, 7)] = 0xFFFF        # already -inf
    scale_code = int(orc.from_f32_16(np.array([scale], np.float32))[0])
    mask = causal_mask16(orc, r1, n, pad) if masked else None
    mshape = (n, r1 + pad, 1, 1) if masked else None
    want = orc.soft_max16(ks16.mode, src, shape, mask, mshape, scale_code, seed=77, nthreads=NT)
    s, w, d = dev16(src), torch.empty(src.size, dtype=torch.int16, device="cuda"), torch.empty(src.size, dtype=torch.int16, device="cuda")
    ks16.soft_max_lns(s, shape, d, w, dev16(mask) if masked else None, mshape, scale_code, 77)
    got = host16(d)
    assert np.array_equal(got, want)


def test_soft_max16_f32(orc, ks16):
    """the kernel_set F32 boundary: F32 logits + F32 ggml mask in, F32 out"""
    rng = np.random.default_rng(8)
    n, r1, r2 = 40, 12, 3
    x = rng.normal(0, 3, (r2, r1, n)).astype(np.float32)
    m = np.zeros((r1, n), np.float32)
    for q in range(r1):
        m[q, q + 1 + n - r1:] = -np.inf
    m[:, 5] = -0.25
    scale = 0.3
    src_c = orc.from_f32_16(x)
    mask_c = orc.mask16(m)
    scale_code = int(orc.from_f32_16(np.array([scale], np.float32))[0])
    want = orc.to_f32_16(orc.soft_max16(ks16.mode, src_c, (n, r1, r2, 1), mask_c, (n, r1, 1, 1), scale_code, seed=5, nthreads=NT))
    xs = torch.from_numpy(x).cuda()
    ms = torch.from_numpy(m).cuda()
    d = torch.empty(x.size, dtype=torch.float32, device="cuda")
    w = torch.empty(x.size, dtype=torch.int16, device="cuda")
    ks16.soft_max(xs, (n, r1, r2, 1), d, w, ms, (n, r1, 1, 1), scale, 5)
    torch.cuda.synchronize()
    assert np.array_equal(d.cpu().numpy().view(np.uint32), want.ravel().view(np.uint32))


# ----------------------------------------------------------------- rms_norm

@pytest.mark.parametrize("ncols,nrows", [(576, 64), (2048, 6), (1, 3), (16, 33)])
def test_rms_norm16(orc, ks16, ncols, nrows):
    rng = np.random.default_rng(ncols + nrows)
    src = codes16(orc, rng, (nrows, ncols), 1.0)
    want = orc.rms_norm16(ks16.mode, src, ncols, nrows, 1e-5, seed=31, nthreads=NT)
    d = torch.empty(src.size, dtype=torch.int16, device="cuda")
    ks16.rms_norm_lns(dev16(src), d, ncols, nrows, 1e-5, 31)
    assert np.array_equal(host16(d), want)


def test_rms_norm16_f32(orc, ks16):
    rng = np.random.default_rng(2)
    x = rng.normal(0, 1, (7, 576)).astype(np.float32)
    want = orc.to_f32_16(orc.rms_norm16(ks16.mode, orc.from_f32_16(x), 576, 7, 1e-5, seed=9, nthreads=NT))
    xs = torch.from_numpy(x).cuda()
    d = torch.empty(x.size, dtype=torch.float32, device="cuda")
    ks16.rms_norm(xs, d, 576, 7, 1e-5, 9)
    torch.cuda.synchronize()
    assert np.array_equal(d.cpu().numpy().view(np.uint32), want.ravel().view(np.uint32))


# ----------------------------------------------------------------- conversions

def test_conversions16(orc, ks16):
    rng = np.random.default_rng(1)
    f = np.concatenate([rng.normal(0, 1, 5000), rng.normal(0, 1e-30, 500), [0.0, -0.0, np.inf, -np.inf, 3e38, -1e-45]])
    f = f.astype(np.float32)
    d = torch.empty(f.size, dtype=torch.int16, device="cuda")
    ks16.to_lns(torch.from_numpy(f).cuda(), d)
    assert np.array_equal(host16(d), orc.from_f32_16(f))
    codes = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    out = torch.empty(65536, dtype=torch.float32, device="cuda")
    ks16.to_f32(dev16(codes), out)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), orc.to_f32_16(codes).view(np.uint32))
    # to_lns_transposed: dst[c * dst_ld + r] = lns(src[r * cols + c])
    rows, cols, ld = 45, 70, 50
    a = rng.normal(0, 0.02, (rows, cols)).astype(np.float32)
    t = torch.zeros(cols * ld, dtype=torch.int16, device="cuda")
    ks16.to_lns_transposed(torch.from_numpy(a).cuda(), t, rows, cols, ld)
    got = host16(t).reshape(cols, ld)[:, :rows]
    assert np.array_equal(got, orc.from_f32_16(a).T)


# ----------------------------------------------------------------- xlns32 (LNSCUDA32)

def codes32(orc, rng, shape, sigma):
    return orc.from_f32_32(rng.normal(0.0, sigma, shape).astype(np.float32))


@pytest.mark.parametrize("K,M,N", [(576, 96, 9), (1, 8, 2), (129, 33, 4), (7, 40, 5), (200, 37, 1),
                                   (40, 2048, 640), (1536, 576, 8)])
def test_mul_mat32(orc, ks32, K, M, N):
    rng = np.random.default_rng(K + M + N)
    w = codes32(orc, rng, (M, K), 0.02)
    x = codes32(orc, rng, (N, K), 1.0)
    want = orc.mul_mat32(w, x, nthreads=NT).ravel()
    out = torch.empty(N * M, dtype=torch.int32, device="cuda")
    ks32.mul_mat_lns(dev32(np.ascontiguousarray(w.T)), dev32(x), out, K, M, N)
    assert np.array_equal(host32(out), want)


def test_mul_mat32_slices_specials_f32(orc, ks32):
    """broadcast slices, special codes (zeros, saturation, cancelling tokens) and F32 output"""
    rng = np.random.default_rng(17)
    ne02, ne03, ne12, ne13 = 1, 2, 3, 2
    M, K, N = 48, 70, 6
    w = codes32(orc, rng, (ne03, ne02, M, K), 0.5)
    x = codes32(orc, rng, (ne13, ne12, N, K), 1.0)
    specials = np.array([0, 0x80000000, 0x7FFFFFFF, 0xFFFFFFFF, 0x40000000, 0xC0000000, 1], np.uint32)
    w.ravel()[rng.integers(0, w.size, 300)] = rng.choice(specials, 300)
    x.ravel()[rng.integers(0, x.size, 100)] = rng.choice(specials, 100)
    x[0, 0, 1] = x[0, 0, 0] ^ 0x80000000
    want = orc.mul_mat32(w, x, slices=(ne02, ne03, ne12, ne13), nthreads=NT).ravel()
    wk = np.ascontiguousarray(np.swapaxes(w, -1, -2))
    out = torch.empty(want.size, dtype=torch.int32, device="cuda")
    ks32.mul_mat_lns(dev32(wk), dev32(x), out, K, M, N, (ne02, ne03, ne12, ne13))
    assert np.array_equal(host32(out), want)
    outf = torch.empty(want.size, dtype=torch.float32, device="cuda")
    ks32.mul_mat(dev32(wk), dev32(x), outf, K, M, N, (ne02, ne03, ne12, ne13))
    torch.cuda.synchronize()
    assert np.array_equal(outf.cpu().numpy().view(np.uint32), orc.to_f32_32(want).view(np.uint32))


@pytest.mark.parametrize("n,r1", [(100, 20), (512, 45), (60000, 3)])   # the last: rows too long for shared memory
def test_soft_max32_rms_norm32(orc, ks32, n, r1):
    rng = np.random.default_rng(4 + n)
    src = codes32(orc, rng, (r1, n), 3.0)
    m = np.zeros((r1, n), np.float32)
    for q in range(r1):
        m[q, q + n - r1 + 1:] = -np.inf
    mask = orc.mask32(m)
    scale_code = int(orc.from_f32_32(np.array([0.125], np.float32))[0])
    want = orc.soft_max32(src, (n, r1, 1, 1), mask, (n, r1, 1, 1), scale_code, nthreads=NT)
    d = torch.empty(src.size, dtype=torch.int32, device="cuda")
    w = torch.empty(src.size, dtype=torch.int32, device="cuda")
    ks32.soft_max_lns(dev32(src), (n, r1, 1, 1), d, w, dev32(mask), (n, r1, 1, 1), scale_code)
    assert np.array_equal(host32(d), want)
    x = codes32(orc, rng, (r1, n), 1.0)
    x.ravel()[:: 17] = 0                                   # zero codes among the squares
    want = orc.rms_norm32(x, n, r1, 1e-5, nthreads=NT)
    d = torch.empty(x.size, dtype=torch.int32, device="cuda")
    ks32.rms_norm_lns(dev32(x), d, n, r1, 1e-5)
    assert np.array_equal(host32(d), want)


def test_conversions32(orc, ks32):
    rng = np.random.default_rng(6)
    f = np.concatenate([rng.normal(0, 1, 20000), rng.normal(0, 1e-40, 300), [0.0, -0.0, 1.0, 2.0, 0.5, np.inf, -3e38]])
    f = f.astype(np.float32)
    d = torch.empty(f.size, dtype=torch.int32, device="cuda")
    ks32.to_lns(torch.from_numpy(f).cuda(), d)
    codes = host32(d)
    assert np.array_equal(codes, orc.from_f32_32(f))
    out = torch.empty(f.size, dtype=torch.float32, device="cuda")
    ks32.to_f32(d, out)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), orc.to_f32_32(codes).view(np.uint32))


def test_errors_are_reported(ks16):
    from lnsb200 import LnsbError
    with pytest.raises(LnsbError):
        ks16.mul_mat_lns(torch.zeros(4, dtype=torch.int16, device="cuda"), torch.zeros(4, dtype=torch.int16, device="cuda"),
                         torch.zeros(4, dtype=torch.int16, device="cuda"), 2, 2, 2, slices=(3, 1, 4, 1))


# ----------------------------------------------------- the latency mat-vec (k_mat_vec_lat)

@pytest.mark.parametrize("fmt", [16, 32])
@pytest.mark.parametrize("K,M,N", [(100, 2000, 3), (1537, 4700, 1), (577, 4000, 4), (33, 1000, 1), (2, 70, 2)])
def test_mat_vec_lat(orc, fmt, K, M, N):
    """sum32 / xlns32 products with few 32-row x 1-token units per SM run the
    producer/chain kernel with 1 .. 4 units per block (a partial last block,
    K not a multiple of the 32-step stage, M not a multiple of 32): bit-exact
    against the oracle"""
    import lnsb200
    rng = np.random.default_rng(K * 7 + M + N)
    if fmt == 16:
        ks = lnsb200.KernelSet(16, "sum32")
        ks.upload_tables()
        w = codes16(orc, rng, (M, K), 0.02)
        x = codes16(orc, rng, (N, K), 1.0)
        want = orc.mul_mat16("sum32", w, x, nthreads=NT).ravel()
        out = torch.empty(N * M, dtype=torch.int16, device="cuda")
        ks.mul_mat_lns(dev16(np.ascontiguousarray(w.T)), dev16(x), out, K, M, N)
        got = host16(out)
    else:
        ks = lnsb200.KernelSet(32, "base")
        ks.upload_tables()
        w = codes32(orc, rng, (M, K), 0.02)
        x = codes32(orc, rng, (N, K), 1.0)
        want = orc.mul_mat32(w, x, nthreads=NT).ravel()
        out = torch.empty(N * M, dtype=torch.int32, device="cuda")
        ks.mul_mat_lns(dev32(np.ascontiguousarray(w.T)), dev32(x), out, K, M, N)
        got = host32(out)
    assert np.array_equal(got, want)


def test_xlns32_conversions_exhaustive(orc, ks32):
    """The xlns32 conversions compute the 2^23-entry mantissa tables' entries in
    double precision (a table read only near the rounding edges): every
    mantissa at an exponent of each sign (float -> xlns32, the +1 of negative
    exponents included) and every fraction field (xlns32 -> float) equal the
    oracle's exact tables"""
    man = np.arange(1 << 23, dtype=np.uint32)
    for ex in (127, 126, 1):                         # 1.m, 0.5 * 1.m (negative log), near the subnormals
        f = ((ex << 23) | man).view(np.float32)
        want = orc.from_f32_32(f)
        out = torch.empty(f.size, dtype=torch.int32, device="cuda")
        ks32.to_lns(torch.from_numpy(f).cuda(), out)
        assert np.array_equal(host32(out), want), ex
    for lg in (0x40000000, 0x3F800000, 0x42000000):  # fraction fields at three log magnitudes
        codes = (np.uint32(lg) + man).astype(np.uint32)
        want = orc.to_f32_32(codes)
        out = torch.empty(codes.size, dtype=torch.float32, device="cuda")
        ks32.to_f32(dev32(codes), out)
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32)), hex(lg)


def test_xlns16_conversion_every_bucket(orc):
    """float -> xlns16: every one of the 131,072 sign / exponent /
    top-mantissa buckets, with its low 15 bits zero, all ones and random,
    gives the oracle's code (zeros, subnormals, infinities and NaNs
    included)"""
    import lnsb200
    ks = lnsb200.KernelSet(16, "base")
    ks.upload_tables()
    rng = np.random.default_rng(21)
    idx = np.arange(1 << 17, dtype=np.uint32)
    for low in (np.zeros_like(idx), np.full_like(idx, 0x7FFF), rng.integers(0, 1 << 15, idx.size).astype(np.uint32)):
        f = ((idx << 15) | low).astype(np.uint32).view(np.float32)
        want = orc.from_f32_16(f)
        out = torch.empty(f.size, dtype=torch.int16, device="cuda")
        ks.to_lns(torch.from_numpy(f).cuda(), out)
        assert np.array_equal(host16(out), want)
