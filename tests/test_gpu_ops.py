"""GPU parity of the model graph's elementwise ops (lnsb_binary / scale /
unary / glu / rope and the F16 conversions) against the CPU oracle, bit for
bit, at the F32 op boundary, in xlns16 (lns-backend/src/lns-ops.cpp:468-599,
786-868, 1199-1281) and xlns32 (lns-backend/src32/lns32-ops.cpp)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def kss():
    import lnsb200
    out = {}
    for fmt in (16, 32):
        out[fmt] = lnsb200.KernelSet(fmt, "base")
        out[fmt].upload_tables()
    return out


@pytest.fixture(scope="module")
def ks(kss):
    return kss[16]


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def f32(rng, shape, sigma=1.0):
    a = rng.normal(0.0, sigma, shape).astype(np.float32)
    flat = a.ravel()
    flat[:: max(1, flat.size // 7)] = 0.0          # zeros among the values
    return a


def same(got, want):
    return np.array_equal(got.view(np.uint32), want.view(np.uint32))


FMTS = pytest.mark.parametrize("fmt", [16, 32])


@FMTS
@pytest.mark.parametrize("op", ["add", "mul", "div"])
@pytest.mark.parametrize("bshape", [(1, 1, 1, 576), (1, 1, 5, 576), (2, 1, 5, 576), (1, 1, 1, 1)])
def test_binary(orc, kss, fmt, op, bshape):
    rng = np.random.default_rng(len(bshape) + bshape[-1] + bshape[-2])
    a = f32(rng, (2, 3, 5, 576))
    b = f32(rng, bshape, 0.5)
    want = orc.binary16(op, a, b, fmt=fmt)
    out = torch.empty(a.size, dtype=torch.float32, device="cuda")
    kss[fmt].binary(op, dev(a), a.shape[::-1], dev(b), b.shape[::-1], out)
    assert same(host(out).reshape(a.shape), want)


@FMTS
@pytest.mark.parametrize("s,b", [(0.125, 0.0), (-3.0, 0.5)])
def test_scale(orc, kss, fmt, s, b):
    rng = np.random.default_rng(3)
    x = f32(rng, (4096,), 2.0)
    out = torch.empty_like(dev(x))
    kss[fmt].scale(dev(x), out, x.size, s, b)
    assert same(host(out), orc.scale16(x, s, b, fmt=fmt))


@FMTS
@pytest.mark.parametrize("op", ["silu", "gelu", "relu", "tanh"])
def test_unary(orc, kss, fmt, op):
    rng = np.random.default_rng(5)
    x = np.concatenate([f32(rng, (8192,), 3.0), np.array([0.0, -0.0, 1e-30, -1e-30, 60.0, -60.0, 1e30, -1e30], np.float32)])
    out = torch.empty_like(dev(x))
    kss[fmt].unary(op, dev(x), out, x.size)
    assert same(host(out), orc.unary16(op, x, fmt=fmt))


@FMTS
@pytest.mark.parametrize("op", ["swiglu", "geglu"])
def test_glu_split_and_fused(orc, kss, fmt, op):
    ks = kss[fmt]
    rng = np.random.default_rng(7)
    nc, nr = 1536, 6
    gate = f32(rng, (nr, nc), 2.0)
    up = f32(rng, (nr, nc), 1.0)
    want = orc.swiglu16(gate, up, fmt=fmt, op=op)
    out = torch.empty((nr, nc), dtype=torch.float32, device="cuda")
    ks.glu(dev(gate), dev(up), nc, nc, out, nc, nr, op=op)
    assert same(host(out), want)
    fused = np.concatenate([gate, up], axis=1)          # [gate | up] per row, stride 2 * nc
    fd = dev(fused)
    ks.glu(fd, fd[:, nc:], 2 * nc, 2 * nc, out, nc, nr, op=op)
    assert same(host(out), want)
    lns = torch.empty((nr, nc), dtype=torch.int16 if fmt == 16 else torch.int32, device="cuda")
    ks.glu_lns(dev(gate), dev(up), nc, nc, lns, nc, nr, op=op)
    codes = orc.from_f32_16(want) if fmt == 16 else orc.from_f32_32(want)
    assert np.array_equal(host(lns).view(codes.dtype), codes)


@FMTS
def test_swiglu_reference_pin(kss, fmt):
    """the reference's printed swiglu (test-lns-backend.cpp run_swiglu_test, the
    LNS16 and LNS32 runs) through the GPU"""
    import json
    import os
    from conftest import ROOT
    p = json.load(open(os.path.join(ROOT, "tests", "golden", "reference_pins.json")))["swiglu"]
    gate = np.array(p["gate"], np.float32).reshape(2, 4)
    up = np.array(p["up"], np.float32).reshape(2, 4)
    out = torch.empty((2, 4), dtype=torch.float32, device="cuda")
    kss[fmt].glu(dev(gate), dev(up), 4, 4, out, 4, 2)
    want = p["out"] if fmt == 16 else p["out_lns32"]
    assert ["%.6f" % v for v in host(out).ravel()] == ["%.6f" % v for v in want]


@FMTS
def test_geglu_tanh_reference_pins(kss, fmt):
    """the reference's printed geglu and tanh (test-lns-backend.cpp
    run_geglu_test / run_tanh_test, the LNS16 and LNS32 runs) through the GPU"""
    import json
    import os
    from conftest import ROOT
    pins = json.load(open(os.path.join(ROOT, "tests", "golden", "reference_pins.json")))
    p = pins["activations"]["lns16" if fmt == 16 else "lns32"]
    gate = np.array(pins["swiglu"]["gate"], np.float32).reshape(2, 4)
    up = np.array(pins["swiglu"]["up"], np.float32).reshape(2, 4)
    out = torch.empty((2, 4), dtype=torch.float32, device="cuda")
    kss[fmt].glu(dev(gate), dev(up), 4, 4, out, 4, 2, op="geglu")
    fmt6 = lambda vs: ["%.6f" % (0.0 if v == 0 else v) for v in vs]
    assert fmt6(host(out).ravel()) == fmt6(p["geglu"])
    x = np.array(p["tanh_in"], np.float32)
    t = torch.empty(8, dtype=torch.float32, device="cuda")
    kss[fmt].unary("tanh", dev(x), t, 8)
    assert fmt6(host(t)) == fmt6(p["tanh"])


@FMTS
@pytest.mark.parametrize("n_dims,neox", [(64, False), (64, True), (32, False)])
def test_rope(orc, kss, fmt, n_dims, neox):
    ks = kss[fmt]
    rng = np.random.default_rng(n_dims + neox)
    hd, nh, nt = 64, 9, 7
    x = f32(rng, (1, nt, nh, hd), 1.0)
    pos = [0, 1, 2, 5, 17, 100, 255]
    cs = orc.rope_cos_sin(pos, n_dims, 100000.0)
    want = orc.rope16(x, cs, n_dims, neox, fmt=fmt)
    out = torch.empty(x.size, dtype=torch.float32, device="cuda")
    ks.rope(dev(x), (hd, nh, nt, 1), dev(cs), n_dims, out, neox=neox)
    assert same(host(out).reshape(x.shape), want)


def test_f16_conversions(ks):
    rng = np.random.default_rng(9)
    x = np.concatenate([rng.normal(0, 3.0, 100000).astype(np.float32),
                        np.array([0.0, -0.0, 65504.0, 7e4, 6e-8, 1e-9, np.inf, -np.inf], np.float32)])
    h = torch.empty(x.size, dtype=torch.int16, device="cuda")
    ks.f32_to_f16(dev(x), h, x.size)
    assert np.array_equal(host(h).view(np.uint16), x.astype(np.float16).view(np.uint16))
    back = torch.empty_like(dev(x))
    ks.f16_to_f32(h, back, x.size)
    assert same(host(back), x.astype(np.float16).astype(np.float32))


def test_invalid(kss):
    import lnsb200
    x = torch.zeros(16, dtype=torch.float32, device="cuda")
    for fmt in (16, 32):
        ks = kss[fmt]
        with pytest.raises(lnsb200.LnsbError):
            ks.binary("add", x, (16, 1, 1, 1), x, (3, 1, 1, 1), x)   # b does not repeat to a
        with pytest.raises(lnsb200.LnsbError):
            ks.glu(x, x, 2, 4, x, 4, 4)                               # gate stride shorter than a row
        assert ks.lib.lnsb_unary(fmt, 4, x.data_ptr(), x.data_ptr(), 16, None) == -1      # no such op: LNSB_E_INVALID


def test_add_latency(kss):
    """lnsb_add_latency: one warp of dependent additions per adder; a plausible
    cycle count per addition (a shared-memory load plus a few integer
    operations), and invalid arguments refused"""
    import torch as _t
    for kind in (0, 1, 2, 3):
        c32 = kss[16].add_latency(kind, 32, 4096)
        c1 = kss[16].add_latency(kind, 1, 4096)
        assert 10 < c1 <= c32 * 1.05 < 1000, (kind, c1, c32)
    out = _t.zeros(2, dtype=_t.int64, device="cuda")
    for args in ((4, 32, 100), (0, 0, 100), (0, 33, 100), (0, 32, 1)):
        assert kss[16].lib.lnsb_add_latency(*args, out.data_ptr(), None) == -1
