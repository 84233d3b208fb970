"""Weights in ggml storage types on the GPU (lnsb_dequantize,
lnsb_to_lns_transposed_typed, the weight cache) against the oracle's
restatement of ggml's block layouts, bit for bit; the reference turns weights
into F32 with ggml's to_float on the host and converts them with
to_lns_transposed (lns-backend/cuda/lns-cuda-context.cpp:163-195, 370-419)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

TYPES = ["f32", "f16", "bf16", "q8_0", "q4_0", "q4_k", "q6_k"]


def random_rows(orc, type, rows, cols, rng):
    """raw uint8 [rows][row_bytes] of a random weight in `type`"""
    qk, bb = orc.BLOCK[type]
    if type in ("f32", "f16", "bf16"):
        v = rng.normal(0, 0.05, (rows, cols)).astype(np.float32)
        if type == "f32":
            return v.view(np.uint8).reshape(rows, -1)
        if type == "f16":
            return v.astype(np.float16).view(np.uint8).reshape(rows, -1)
        return (v.view(np.uint32) >> 16).astype(np.uint16).view(np.uint8).reshape(rows, -1)
    raw = rng.integers(0, 256, (rows, (cols // qk) * bb), dtype=np.uint8)
    nb = cols // qk
    for i in range(nb):                                  # sane f16 scales: finite, about 1e-3 .. 1e-1
        for off in ({"q8_0": [0], "q4_0": [0], "q4_k": [0, 2], "q6_k": [208]}[type]):
            d = rng.uniform(1e-3, 1e-1, rows).astype(np.float16).view(np.uint8).reshape(rows, 2)
            raw[:, i * bb + off:i * bb + off + 2] = d
    return raw


@pytest.fixture(scope="module")
def kss():
    import lnsb200
    out = {}
    for fmt in (16, 32):
        out[fmt] = lnsb200.KernelSet(fmt, "base")
        out[fmt].upload_tables()
    return out


@pytest.mark.parametrize("type", TYPES)
def test_dequantize(orc, kss, type):
    rng = np.random.default_rng(len(type) * 17)
    rows, cols = 37, 512
    raw = random_rows(orc, type, rows, cols, rng)
    assert raw.shape[1] == kss[16].type_row_bytes(type, cols)
    out = torch.empty(rows * cols, dtype=torch.float32, device="cuda")
    kss[16].dequantize(type, torch.from_numpy(raw).cuda(), out, rows, cols)
    torch.cuda.synchronize()
    want = orc.dequant(type, raw, rows, cols)
    assert np.array_equal(out.cpu().numpy().reshape(rows, cols).view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("fmt", [16, 32])
@pytest.mark.parametrize("type", TYPES)
def test_to_lns_transposed_typed(orc, kss, fmt, type):
    rng = np.random.default_rng(len(type) + fmt)
    rows, cols = 45, 768
    raw = random_rows(orc, type, rows, cols, rng)
    it = torch.int16 if fmt == 16 else torch.int32
    dst = torch.empty(cols * rows, dtype=it, device="cuda")
    kss[fmt].to_lns_transposed_typed(type, torch.from_numpy(raw).cuda(), dst, rows, cols, rows)
    torch.cuda.synchronize()
    f = orc.dequant(type, raw, rows, cols)
    want = (orc.from_f32_16(f) if fmt == 16 else orc.from_f32_32(f)).T.reshape(-1)
    got = dst.cpu().numpy().view(np.uint16 if fmt == 16 else np.uint32)
    assert np.array_equal(got, want)


def _specials(type, raw, rng):
    """plants zeros, subnormals, infinities, NaNs and extremes in element-type rows"""
    if type == "f16":
        pats = np.array([0x0000, 0x8000, 0x0001, 0x83FF, 0x0400, 0x7BFF, 0xFBFF, 0x7C00, 0xFC00, 0x7E00, 0x3C00, 0xBC00],
                        np.uint16)
        v = raw.view(np.uint16)
    elif type == "bf16":
        pats = np.array([0x0000, 0x8000, 0x0001, 0x807F, 0x0080, 0x7F7F, 0xFF7F, 0x7F80, 0xFF80, 0x7FC0, 0x3F80, 0x0100],
                        np.uint16)
        v = raw.view(np.uint16)
    elif type == "f32":
        pats = np.array([0x00000000, 0x80000000, 0x00000001, 0x807FFFFF, 0x00800000, 0x7F7FFFFF, 0xFF7FFFFF, 0x7F800000,
                         0xFF800000, 0x7FC00000, 0x3F800000, 0x01000000], np.uint32)
        v = raw.view(np.uint32)
    else:
        return raw
    idx = rng.integers(0, v.size, 400)
    v.reshape(-1)[idx] = rng.choice(pats, 400)
    return raw


@pytest.mark.parametrize("type,rows,cols,dst_ld,misalign", [
    ("f16", 130, 576, 136, 0),     # 16-byte stores, a partial row tile and a partial column tile
    ("f16", 64, 512, 64, 2),       # source not 16-byte aligned: byte staging
    ("bf16", 129, 300, 129, 0),
    ("f32", 70, 200, 72, 0),
    ("q8_0", 96, 576, 96, 0),
    ("q4_0", 65, 288, 72, 0),
    ("q4_k", 70, 1024, 72, 0),
    ("q6_k", 70, 2048, 72, 0),     # 16-byte rows: staged windows that start inside a 16-byte piece
    ("q6_k", 33, 768, 40, 0),
])
def test_to_lns_transposed_typed_tiles(orc, kss, type, rows, cols, dst_ld, misalign):
    """the tiled xlns16 conversion: every tile edge, both copy paths, both
    store paths, and (element types) zeros, subnormals, infinities, NaNs"""
    rng = np.random.default_rng(rows * 7 + cols)
    raw = _specials(type, np.ascontiguousarray(random_rows(orc, type, rows, cols, rng)), rng)
    buf = torch.zeros(raw.size + 16, dtype=torch.uint8, device="cuda")
    buf[misalign:misalign + raw.size] = torch.from_numpy(raw.reshape(-1)).cuda()
    dst = torch.full((cols * dst_ld,), 0x1234, dtype=torch.int16, device="cuda")
    kss[16].to_lns_transposed_typed(type, buf[misalign:], dst, rows, cols, dst_ld)
    torch.cuda.synchronize()
    want = orc.from_f32_16(orc.dequant(type, raw, rows, cols)).T                       # [cols][rows]
    got = dst.cpu().numpy().view(np.uint16).reshape(cols, dst_ld)
    assert np.array_equal(got[:, :rows], want)
    assert np.all(got[:, rows:] == 0x1234)                                                # padding untouched


def image_f32(ks, addr, n):
    """the F32 decode of n LNS codes at a device address (lnsb_to_f32)"""
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    assert ks.lib.lnsb_to_f32(ks.fmt, addr, out.data_ptr(), n, None) == 0
    torch.cuda.synchronize()
    return out.cpu().numpy()


def test_weight_cache(orc, kss):
    import lnsb200
    ks = kss[16]
    rng = np.random.default_rng(3)
    rows, cols = 300, 512
    raw = random_rows(orc, "q4_k", rows, cols, rng)
    want = orc.to_f32_16(orc.from_f32_16(orc.dequant("q4_k", raw, rows, cols)).T.reshape(-1))
    nbytes = rows * cols * 2
    dsrc = torch.from_numpy(raw).cuda()
    c = lnsb200.WeightCache(ks, budget=2 * nbytes)
    a1 = c.get(dsrc, "q4_k", rows, cols)
    assert c.get(dsrc, "q4_k", rows, cols) == a1
    assert c.stats() == {"entries": 1, "used": nbytes, "budget": 2 * nbytes}
    assert np.array_equal(image_f32(ks, a1, rows * cols).view(np.uint32), want.view(np.uint32))
    # host rows (numpy): staged to the device, their own entry
    a2 = c.get(raw, "q4_k", rows, cols)
    assert a2 != a1 and c.stats()["entries"] == 2
    assert np.array_equal(image_f32(ks, a2, rows * cols).view(np.uint32), want.view(np.uint32))
    # over budget: the image goes to the caller's scratch and is not cached
    scratch = torch.empty(rows * cols, dtype=torch.int16, device="cuda")
    dsrc2 = dsrc.clone()
    assert c.get(dsrc2, "q4_k", rows, cols, scratch=scratch) == scratch.data_ptr()
    assert c.stats()["entries"] == 2
    assert np.array_equal(image_f32(ks, scratch.data_ptr(), rows * cols).view(np.uint32), want.view(np.uint32))
    with pytest.raises(lnsb200.LnsbError):               # over budget and no scratch
        c.get(dsrc2, "q4_k", rows, cols)
    c.close()


def test_weight_cache_xlns32_host_rows(orc, kss):
    import lnsb200
    ks = kss[32]
    rng = np.random.default_rng(4)
    rows, cols = 64, 256
    raw = random_rows(orc, "q6_k", rows, cols, rng)
    want = orc.to_f32_32(orc.from_f32_32(orc.dequant("q6_k", raw, rows, cols)).T.reshape(-1))
    c = lnsb200.WeightCache(ks, budget=1 << 20)
    addr = c.get(raw, "q6_k", rows, cols)
    assert np.array_equal(image_f32(ks, addr, rows * cols).view(np.uint32), want.view(np.uint32))
    tiny = lnsb200.WeightCache(ks, budget=0)             # nothing fits: always the scratch
    scratch = torch.empty(rows * cols, dtype=torch.int32, device="cuda")
    assert tiny.get(raw, "q6_k", rows, cols, scratch=scratch) == scratch.data_ptr()
    assert tiny.stats()["entries"] == 0
    assert np.array_equal(image_f32(ks, scratch.data_ptr(), rows * cols).view(np.uint32), want.view(np.uint32))
    c.close()
    tiny.close()


def test_typed_errors(kss):
    import lnsb200
    ks = kss[16]
    z = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    d = torch.zeros(4096, dtype=torch.int16, device="cuda")
    with pytest.raises(lnsb200.LnsbError):
        ks.to_lns_transposed_typed(3, z, d, 4, 32, 4)        # Q4_1: not supported
    with pytest.raises(lnsb200.LnsbError):
        ks.to_lns_transposed_typed("q4_k", z, d, 4, 128, 4)  # half a Q4_K block
    assert ks.type_row_bytes("q6_k", 512) == 420 and ks.type_row_bytes("q4_k", 100) == 0


def test_weight_cache_allocation_failure(orc, kss, monkeypatch):
    """An out-of-memory allocation in the cache (injected on the host,
    LNSB_WEIGHT_CACHE_FAIL_ALLOCS) leaves no sticky error: the image goes to
    scratch, or the call reports LNSB_E_TOO_LARGE without scratch, nothing is
    cached, and the next allocation and a mul_mat afterwards succeed."""
    import lnsb200
    ks = kss[16]
    rng = np.random.default_rng(5)
    rows, cols = 64, 256
    raw = random_rows(orc, "q4_k", rows, cols, rng)
    want = orc.to_f32_16(orc.from_f32_16(orc.dequant("q4_k", raw, rows, cols)).T.reshape(-1))
    dsrc = torch.from_numpy(raw).cuda()
    monkeypatch.setenv("LNSB_WEIGHT_CACHE_FAIL_ALLOCS", "2")
    c = lnsb200.WeightCache(ks, budget=1 << 30)
    scratch = torch.empty(rows * cols, dtype=torch.int16, device="cuda")
    assert c.get(dsrc, "q4_k", rows, cols, scratch=scratch) == scratch.data_ptr()     # failure 1: to scratch
    assert c.stats()["entries"] == 0
    assert np.array_equal(image_f32(ks, scratch.data_ptr(), rows * cols).view(np.uint32), want.view(np.uint32))
    with pytest.raises(lnsb200.LnsbError):                                              # failure 2: no scratch
        c.get(dsrc, "q4_k", rows, cols)
    a = c.get(dsrc, "q4_k", rows, cols)                                                 # allocations work again
    assert c.stats()["entries"] == 1 and a != scratch.data_ptr()
    assert np.array_equal(image_f32(ks, a, rows * cols).view(np.uint32), want.view(np.uint32))
    c.close()
    # the context is clean: an ordinary mul_mat runs bit-exact afterwards
    K, M, N = 64, 16, 3
    w = orc.from_f32_16(rng.normal(0, 0.1, (M, K)).astype(np.float32))
    x = orc.from_f32_16(rng.normal(0, 1, (N, K)).astype(np.float32))
    wd = torch.from_numpy(np.ascontiguousarray(w.T).view(np.int16)).cuda()
    xd = torch.from_numpy(x.view(np.int16)).cuda()
    out = torch.empty(N * M, dtype=torch.int16, device="cuda")
    ks.mul_mat_lns(wd, xd, out, K, M, N)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint16).reshape(N, M), orc.mul_mat16(ks.mode, w, x, seed=7))
