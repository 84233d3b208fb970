"""GPU == oracle at BASELINE configs[4]'s full size (the sum32 sweep's largest
shape: 8192 weight rows, K = 14336, N in {1, 16, 128}), in every summation
mode and in xlns32.

The oracle is too slow for the whole product (15 G additions at N = 128), so
the full-size result is checked two ways:
- sampled rows: contiguous row blocks at the start, in the middle and at the
  end of the matrix are recomputed by the oracle over every token.  A Monte
  block starting at row m0 starts its LFSR m0 * N * (K - 1) draws after the
  op's seed, the jump of the CPU loop order (lns-backend/src/lns-ops.cpp:
  342-372; draw accounting lns-backend/cuda/lns-cuda-kernels.cuh:107-115);
- row-shard invariance over the whole output: the upper half of the rows,
  run as its own mul_mat with the shard's Monte seed, gives exactly the upper
  half of the full result (every output is its own chain, so splitting rows
  never changes a bit -- the property the multi-GPU row sharding relies on).
Results are compared as integer codes, as every parity test here is.
"""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

MODES = ("base", "monte", "monte_bylpvip", "lpvip", "sum32")
NT = os.cpu_count() or 1
K, M = 14336, 8192
BLOCKS = ((0, 8), (4093, 8), (8184, 8))      # (first row, rows): start, an unaligned middle block, end


@pytest.fixture(scope="module")
def data(orc):
    """configs[4] inputs (numpy default_rng(3)): W 8192 x K N(0, 0.02), X 128 x K N(0, 1)"""
    rng = np.random.default_rng(3)
    w = rng.normal(0.0, 0.02, (M, K)).astype(np.float32)
    x = rng.normal(0.0, 1.0, (128, K)).astype(np.float32)
    return w, x


@pytest.fixture(scope="module")
def codes16(orc, data):
    w, x = data
    wc, xc = orc.from_f32_16(w), orc.from_f32_16(x)
    wk = torch.from_numpy(wc.view(np.int16)).cuda().t().contiguous()        # k-major [K][M] on the device
    return wc, xc, wk


def _check_blocks(got, want_of_block, N):
    for m0, r in BLOCKS:
        want = want_of_block(m0, r)                                         # [N][r]
        blk = got.reshape(N, M)[:, m0:m0 + r]
        bad = np.argwhere(blk != want)
        assert bad.size == 0, "rows %d..%d: first mismatch at token %d row %d" % (m0, m0 + r, bad[0][0], m0 + bad[0][1])


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("N", [1, 16, 128])
def test_configs4_full_size(orc, codes16, mode, N):
    from lnsb200 import KernelSet
    ks = KernelSet(16, mode)
    ks.upload_tables()
    wc, xc, wk = codes16
    xs = np.ascontiguousarray(xc[:N])
    xd = torch.from_numpy(xs.view(np.int16)).cuda()
    out = torch.empty(N * M, dtype=torch.int16, device="cuda")
    ks.mul_mat_lns(wk, xd, out, K, M, N, monte_seed=7)
    torch.cuda.synchronize()
    got = out.cpu().numpy().view(np.uint16)

    def want_of_block(m0, r):
        seed = orc.lfsr_jump(7, m0 * N * (K - 1))
        return orc.mul_mat16(mode, wc[m0:m0 + r], xs, seed=seed, nthreads=NT).reshape(N, r)
    _check_blocks(got, want_of_block, N)

    # the upper half of the rows as its own op: the same bits
    h = M // 2
    seed_h = orc.lfsr_jump(7, h * N * (K - 1))
    wk_h = wk[:, h:].contiguous()
    out_h = torch.empty(N * h, dtype=torch.int16, device="cuda")
    ks.mul_mat_lns(wk_h, xd, out_h, K, h, N, monte_seed=seed_h)
    torch.cuda.synchronize()
    assert np.array_equal(out_h.cpu().numpy().view(np.uint16).reshape(N, h), got.reshape(N, M)[:, h:])


def test_configs4_full_size_xlns32(orc, data):
    """the same shape (N = 128) in xlns32 (LNSCUDA32), sampled rows"""
    from lnsb200 import KernelSet
    ks = KernelSet(32, "base")
    ks.upload_tables()
    w, x = data
    N = 128
    wc, xc = orc.from_f32_32(w), orc.from_f32_32(x)
    wk = torch.from_numpy(wc.view(np.int32)).cuda().t().contiguous()
    xd = torch.from_numpy(xc.view(np.int32)).cuda()
    out = torch.empty(N * M, dtype=torch.int32, device="cuda")
    ks.mul_mat_lns(wk, xd, out, K, M, N)
    torch.cuda.synchronize()
    got = out.cpu().numpy().view(np.uint32)
    _check_blocks(got, lambda m0, r: orc.mul_mat32(wc[m0:m0 + r], xc, nthreads=NT).reshape(N, r), N)
