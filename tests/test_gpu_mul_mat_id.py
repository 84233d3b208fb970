"""MUL_MAT_ID (the expert-selected product, lns-backend/src/lns-ops.cpp:394-462)
on the GPU against the oracle, bit for bit, in every summation-mode build and
in xlns32: slot-based broadcast of the activation rows (ne11 < n_used),
repeated experts, K = 1, ragged M, Monte chain offsets in the CPU loop order,
F32 and LNS outputs, and out-of-range ids (counted, zero code)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

MODES = ("base", "monte", "monte_bylpvip", "lpvip", "sum32")


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


def run(ks, orc, fmt, n_expert, K, M, n_tokens, n_used, ne11, seed=7, bad_slot=None, f32=False, specials=False):
    rng = np.random.default_rng(K * 131 + M * 7 + n_tokens + n_used)
    tof = orc.from_f32_16 if fmt == 16 else orc.from_f32_32
    w_rows = tof(rng.normal(0, 0.02, (n_expert, M, K)).astype(np.float32))      # [e][m][k]
    x = tof(rng.normal(0, 1, (n_tokens, ne11, K)).astype(np.float32))
    if specials:                                          # zeros, saturations, exact opposites along K
        sp = np.array([0x0000, 0x8000, 0x7FFF, 0xFFFF, 0x0001], np.uint16)
        w_rows.ravel()[rng.integers(0, w_rows.size, 200)] = rng.choice(sp, 200)
        x.ravel()[rng.integers(0, x.size, 20)] = rng.choice(sp, 20)
        x[0, 0, K // 2] = x[0, 0, K // 2 - 1] ^ 0x8000
    ids = rng.integers(0, n_expert, (n_tokens, n_used)).astype(np.int32)
    if n_tokens > 1:
        ids[1, :] = ids[0, 0]                               # one expert in every slot of a token
    if bad_slot is not None:
        ids[bad_slot] = n_expert + 3
    want, bad = orc.mul_mat_id(fmt, ks.mode if fmt == 16 else None, w_rows, x, ids, seed=seed, nthreads=8)
    it = torch.int16 if fmt == 16 else torch.int32
    view = np.uint16 if fmt == 16 else np.uint32
    wk = np.ascontiguousarray(np.transpose(w_rows, (0, 2, 1)))                  # k-major per expert: [e][k][m]
    dw = torch.from_numpy(wk.view(np.int16 if fmt == 16 else np.int32)).cuda()
    dx = torch.from_numpy(np.ascontiguousarray(x).view(np.int16 if fmt == 16 else np.int32)).cuda()
    di = torch.from_numpy(ids).cuda()
    ks.mul_mat_id_bad_ids()                                # clear the counter
    if f32:
        out = torch.empty(n_tokens * n_used * M, dtype=torch.float32, device="cuda")
        ks.mul_mat_id(dw, dx, di, out, K, M, n_expert, ne11, n_used, n_tokens, monte_seed=seed)
        torch.cuda.synchronize()
        got = out.cpu().numpy().reshape(n_tokens, n_used, M)
        wantf = (orc.to_f32_16 if fmt == 16 else orc.to_f32_32)(want)
        return np.array_equal(got.view(np.uint32), wantf.view(np.uint32)), ks.mul_mat_id_bad_ids(), bad
    out = torch.empty(n_tokens * n_used * M, dtype=it, device="cuda")
    ks.mul_mat_id_lns(dw, dx, di, out, K, M, n_expert, ne11, n_used, n_tokens, monte_seed=seed)
    torch.cuda.synchronize()
    got = out.cpu().numpy().view(view).reshape(n_tokens, n_used, M)
    return np.array_equal(got, want), ks.mul_mat_id_bad_ids(), bad


@pytest.mark.parametrize("n_expert,K,M,n_tokens,n_used,ne11", [
    (8, 576, 1408, 1, 2, 1),       # decode: one token, two experts
    (8, 576, 96, 5, 4, 2),         # slot-based broadcast over two activation rows
    (4, 1, 33, 3, 2, 1),           # K = 1
    (6, 129, 77, 4, 3, 3),         # ragged M, one activation row per slot
])
def test_mul_mat_id16(orc, ks16, n_expert, K, M, n_tokens, n_used, ne11):
    ok, bad_gpu, bad_orc = run(ks16, orc, 16, n_expert, K, M, n_tokens, n_used, ne11, seed=0xB403)
    assert ok and bad_gpu == bad_orc == 0


def test_mul_mat_id16_special_codes(orc, ks16):
    """zeros, saturated codes and cancelling terms part-way along the chains:
    in base mode they move a chain from the key form to packed codes and
    back, bit-exact either way"""
    ok, bad_gpu, bad_orc = run(ks16, orc, 16, 6, 300, 200, 4, 2, 1, seed=5, specials=True)
    assert ok and bad_gpu == bad_orc == 0


def test_mul_mat_id16_f32_and_bad_ids(orc, ks16):
    ok, bad_gpu, bad_orc = run(ks16, orc, 16, 4, 200, 70, 3, 2, 1, f32=True, bad_slot=(2, 1))
    assert ok and bad_gpu == bad_orc == 1


@pytest.mark.parametrize("n_expert,K,M,n_tokens,n_used,ne11", [(8, 576, 320, 2, 2, 1), (3, 65, 40, 3, 2, 2)])
def test_mul_mat_id32(orc, ks32, n_expert, K, M, n_tokens, n_used, ne11):
    ok, bad_gpu, bad_orc = run(ks32, orc, 32, n_expert, K, M, n_tokens, n_used, ne11)
    assert ok and bad_gpu == bad_orc == 0
    ok, bad_gpu, bad_orc = run(ks32, orc, 32, n_expert, K, M, n_tokens, n_used, ne11, f32=True, bad_slot=(0, 1))
    assert ok and bad_gpu == bad_orc == 1


def test_mul_mat_id_invalid(ks16):
    import lnsb200
    z = torch.zeros(64, dtype=torch.int16, device="cuda")
    ids = torch.zeros(4, dtype=torch.int32, device="cuda")
    with pytest.raises(lnsb200.LnsbError):                 # n_used % ne11 != 0
        ks16.mul_mat_id_lns(z, z, ids, z, 4, 4, 1, 3, 2, 2)
    assert ks16.mul_mat_id_draws(10, 4, 2, 3) == (3 * 2 * 4 * 9 if ks16.mode in ("monte", "monte_bylpvip") else 0)


def test_mul_mat_id_k0_and_empty(orc, ks16):
    """K = 0 gives the zero code (the oracle's empty chain); no tokens is a no-op"""
    z = torch.zeros(64, dtype=torch.int16, device="cuda")
    ids = torch.zeros(4, dtype=torch.int32, device="cuda")
    out = torch.full((2 * 2 * 8,), 0x1234, dtype=torch.int16, device="cuda")
    ks16.mul_mat_id_lns(z, z, ids, out, 0, 8, 1, 1, 2, 2)
    torch.cuda.synchronize()
    assert (out.cpu().numpy() == 0).all()
    ks16.mul_mat_id_lns(z, z, ids, out, 4, 8, 1, 1, 2, 0)     # n_tokens = 0
