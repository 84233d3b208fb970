"""graph_compute of the ggml backend's host layer (lnsb_graph_compute) on the
GPU: a LLaMA-style block written as ggml-like nodes -- rms_norm, the norm
weight, an F16 weight matrix (weight cache), rope with I32 positions, the
attention scores through a permuted F16 KV-cache view with GQA broadcast (the
reference's parity case lns-backend/tests/test-lns-cuda-parity.cpp:255-366),
the softmax with a padded mask, an F32 matrix and a Q8_0 matrix, fused
swiglu, silu, add, scale -- every node's result bit for bit against the CPU
oracle run op by op on the same F32 inputs; the same graph over host
buffers (the reference's per-op upload / download) equal to the device run;
unsupported and skipped nodes."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

T, D, H, HD, HKV, FF, NKV = 5, 64, 4, 16, 2, 96, 7


def q8_0_blocks(rng, rows, cols):
    """random Q8_0 rows: per 32 values an f16 scale then 32 int8 quants"""
    nb = cols // 32
    raw = np.zeros((rows, nb, 34), np.uint8)
    raw[:, :, 0:2] = rng.uniform(1e-3, 2e-3, (rows, nb)).astype(np.float16).view(np.uint8).reshape(rows, nb, 2)
    raw[:, :, 2:] = rng.integers(-127, 128, (rows, nb, 32)).astype(np.int8).view(np.uint8)
    return raw.reshape(rows, nb * 34)


def inputs(seed=0):
    rng = np.random.default_rng(seed)
    f = lambda *s, sd=1.0: rng.normal(0, sd, s).astype(np.float32)   # noqa: E731
    kv = rng.normal(0, 1, (8, HKV * HD)).astype(np.float16)           # the K cache, 8 slots, NKV used
    mask = np.full((8, 16), -np.inf, np.float32)                       # [T (padded to 8)][16 keys, padded]
    for t in range(T):
        mask[t, :NKV - T + t + 1] = 0.0
    return dict(x=f(T, D), nw=f(D, sd=0.5) + 1.0, wq=f(D, D, sd=0.05).astype(np.float16),
                wup=f(2 * FF, D, sd=0.05), q8=q8_0_blocks(rng, 32, D), kv=kv, mask=mask,
                pos=np.arange(NKV - T, NKV, dtype=np.int32))


def build(G, a, dev):
    """the block's nodes over the arrays of `a` (torch tensors on the device, or
    numpy arrays on the host); returns (nodes in order, {name: result array})"""
    out = {}

    def mk(name, shape, dtype=np.float32):
        arr = torch.zeros(shape, dtype=getattr(torch, np.dtype(dtype).name), device="cuda") if dev \
            else np.zeros(shape, dtype)
        out[name] = arr
        return arr

    x = G.tensor(a["x"], name="inp_embd")
    nw = G.tensor(a["nw"], name="blk.0.attn_norm.weight")
    wq = G.tensor(a["wq"], name="blk.0.attn_q.weight", flags=G.FLAG_WEIGHTS)
    wup = G.tensor(a["wup"], name="blk.0.ffn_up.weight", flags=G.FLAG_WEIGHTS)
    q8 = G.tensor(None, type="q8_0", ne=[D, 32, 1, 1], nb=[34, 68, 68 * 32, 68 * 32],
                  data=a["q8"].data_ptr() if dev else a["q8"].ctypes.data, name="blk.0.ffn_q8.weight",
                  flags=G.FLAG_WEIGHTS)
    pos = G.tensor(a["pos"], name="inp_pos")
    C = G.FLAG_COMPUTE
    n1 = G.tensor(mk("norm", (T, D)), op="RMS_NORM", src=(x,), params=(1e-5,), name="norm-0", flags=C)
    n2 = G.tensor(mk("attn_norm", (T, D)), op="MUL", src=(n1, nw), name="attn_norm-0", flags=C)
    n3 = G.tensor(mk("Qcur", (T, D)), op="MUL_MAT", src=(wq, n2), name="Qcur-0", flags=C)
    q3 = G.tensor(out["Qcur"].view(T, H, HD) if dev else out["Qcur"].reshape(T, H, HD), op="VIEW", src=(n3,),
                  name="Qcur-0 (view)", flags=C)
    n4 = G.tensor(mk("Qrope", (T, H, HD)), op="ROPE", src=(q3, pos),
                  params=(0, HD, 0, 0, 0, 10000.0, 1.0, 0.0, 1.0), name="Qcur-0 (rope)", flags=C)
    # the K cache [slot][kv head][dim] as ne (dim, key, kv head): a permuted view
    kvv = G.tensor(None, type="f16", ne=[HD, NKV, HKV, 1], nb=[2, HKV * HD * 2, HD * 2, 8 * HKV * HD * 2],
                   data=a["kv"].data_ptr() if dev else a["kv"].ctypes.data, name="cache_k_l0 (view)")
    # q as ne (dim, token, head): a permuted view of the roped q
    qp = G.tensor(None, type="f32", ne=[HD, T, H, 1], nb=[4, H * HD * 4, HD * 4, T * H * HD * 4],
                  data=out["Qrope"].data_ptr() if dev else out["Qrope"].ctypes.data, name="q (permuted)",
                  op="PERMUTE", src=(n4,), flags=C)
    n5 = G.tensor(mk("kq", (H, T, NKV)), op="MUL_MAT", src=(kvv, qp), name="kq-0", flags=C)
    mk_ = G.tensor(a["mask"], name="KQ_mask")
    n6 = G.tensor(mk("kq_soft_max", (H, T, NKV)), op="SOFT_MAX", src=(n5, mk_), params=(0.25, 0.0),
                  name="kq_soft_max-0", flags=C)
    n7 = G.tensor(mk("up", (T, 2 * FF)), op="MUL_MAT", src=(wup, n2), name="ffn_up-0", flags=C)
    n8 = G.tensor(mk("swiglu", (T, FF)), op="GLU", src=(n7,), params=(G.GLU["swiglu"], 0), name="ffn_swiglu-0", flags=C)
    n9 = G.tensor(mk("q8", (T, 32)), op="MUL_MAT", src=(q8, n2), name="ffn_q8-0", flags=C)
    n10 = G.tensor(mk("silu", (T, D)), op="UNARY", src=(n3,), params=(G.UNARY["silu"],), name="silu-0", flags=C)
    n11 = G.tensor(mk("add", (T, D)), op="ADD", src=(x, n3), name="attn_out-0", flags=C)
    n12 = G.tensor(mk("scale", (T, D)), op="SCALE", src=(n11,), params=(0.5, 0.25), name="scaled-0", flags=C)
    return [n1, n2, n3, q3, n4, qp, n5, n6, n7, n8, n9, n10, n11, n12], out


def expected(orc, a, mode, fmt):
    """the block op by op through the CPU oracle, from the same F32 inputs"""
    c16 = fmt == 16
    to_c = orc.from_f32_16 if c16 else orc.from_f32_32
    to_f = orc.to_f32_16 if c16 else orc.to_f32_32

    def mm(w_rows, x_rows, slices=(1, 1, 1, 1)):
        if c16:
            return to_f(orc.mul_mat16(mode, to_c(w_rows), to_c(x_rows), slices=slices, seed=0, nthreads=8))
        return to_f(orc.mul_mat32(to_c(w_rows), to_c(x_rows), slices=slices, nthreads=8))

    e = {}
    x = a["x"]
    rms = orc.rms_norm16(mode, to_c(x).ravel(), D, T, 1e-5) if c16 else orc.rms_norm32(to_c(x).ravel(), D, T, 1e-5)
    e["norm"] = to_f(rms).reshape(T, D)
    e["attn_norm"] = orc.binary16("mul", e["norm"], a["nw"].reshape(1, D), fmt=fmt)
    e["Qcur"] = mm(a["wq"].astype(np.float32), e["attn_norm"]).reshape(T, D)
    cs = orc.rope_cos_sin(list(a["pos"]), HD, 10000.0)
    e["Qrope"] = orc.rope16(e["Qcur"].reshape(1, T, H, HD), cs, HD, False, fmt=fmt).reshape(T, H, HD)
    k = a["kv"][:NKV].astype(np.float32).reshape(NKV, HKV, HD).transpose(1, 0, 2)       # [kv head][key][dim]
    q = e["Qrope"].transpose(1, 0, 2)                                                    # [head][token][dim]
    e["kq"] = mm(np.ascontiguousarray(k).reshape(1, HKV, NKV, HD), np.ascontiguousarray(q).reshape(1, H, T, HD),
                 slices=(HKV, 1, H, 1)).reshape(H, T, NKV)
    m = np.ascontiguousarray(a["mask"][:, :NKV])
    sc = int(to_c(np.array([0.25], np.float32))[0])
    if c16:
        sm = orc.soft_max16(mode, to_c(e["kq"]).ravel(), (NKV, T, H, 1), orc.mask16(m).ravel(), (NKV, 8, 1, 1), sc, seed=0)
    else:
        sm = orc.soft_max32(to_c(e["kq"]).ravel(), (NKV, T, H, 1), orc.mask32(m).ravel(), (NKV, 8, 1, 1), sc)
    e["kq_soft_max"] = to_f(sm).reshape(H, T, NKV)
    e["up"] = mm(a["wup"], e["attn_norm"]).reshape(T, 2 * FF)
    e["swiglu"] = orc.swiglu16(np.ascontiguousarray(e["up"][:, :FF]), np.ascontiguousarray(e["up"][:, FF:]), fmt=fmt)
    e["q8"] = mm(orc.dequant("q8_0", a["q8"], 32, D), e["attn_norm"]).reshape(T, 32)
    e["silu"] = orc.unary16("silu", e["Qcur"], fmt=fmt)
    e["add"] = orc.binary16("add", x, e["Qcur"], fmt=fmt)
    e["scale"] = orc.scale16(e["add"], 0.5, 0.25, fmt=fmt)
    return e


def dev_arrays(a):
    return {k: torch.from_numpy(v).cuda() for k, v in a.items()}


@pytest.mark.parametrize("fmt,mode", [(16, "base"), (16, "sum32"), (16, "monte"), (32, "base")])
def test_graph_compute_matches_the_oracle_op_by_op(orc, fmt, mode):
    from lnsb200 import graph as G
    a = inputs()
    if mode == "monte":
        assert G.lib(mode).lnsb_monte_set_state(7) == 0
    g = G.Graph(fmt, mode)
    nodes, out = build(G, dev_arrays(a), True)
    st, failed = g.compute(nodes)
    assert (st, failed) == (0, -1)
    torch.cuda.synchronize()
    if mode == "monte":
        return                  # the draws follow the library's LFSR state: parity covered by the op tests
    want = expected(orc, a, mode, fmt)
    for name, arr in out.items():
        got = arr.cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want[name].reshape(got.shape).view(np.uint32)), name
    g.close()


def test_graph_compute_over_host_buffers_equals_the_device_run():
    """host-memory tensors (the reference's CPU buffer type): each op uploads
    its operands and downloads its result, and gives the device run's bits"""
    from lnsb200 import graph as G
    a = inputs(1)
    g = G.Graph(16, "sum32")
    nodes_d, out_d = build(G, dev_arrays(a), True)
    assert g.compute(nodes_d) == (0, -1)
    host = {k: np.ascontiguousarray(v) for k, v in a.items()}
    nodes_h, out_h = build(G, host, False)
    assert g.compute(nodes_h) == (0, -1)
    torch.cuda.synchronize()
    for name in out_d:
        assert np.array_equal(out_d[name].cpu().numpy().view(np.uint32), out_h[name].view(np.uint32)), name
    g.close()


def test_graph_compute_refuses_and_skips():
    """a node without a kernel stops the walk with LNSB_E_UNSUPPORTED and its
    index (the reference aborts); nodes without the compute flag, views and
    empty tensors are skipped"""
    from lnsb200 import graph as G
    g = G.Graph(16, "base")
    x = torch.zeros((4, 8), dtype=torch.float32, device="cuda")
    y = torch.full((4, 8), 7.0, dtype=torch.float32, device="cuda")
    src = G.tensor(x)
    skipped = G.tensor(y, op="SCALE", src=(src,), params=(2.0, 0.0))                 # no compute flag
    view = G.tensor(y, op="VIEW", src=(src,), flags=G.FLAG_COMPUTE)
    empty = G.tensor(torch.zeros((0, 8), device="cuda"), op="SCALE", src=(G.tensor(torch.zeros((0, 8), device="cuda")),),
                     params=(2.0, 0.0), flags=G.FLAG_COMPUTE)
    rows = G.tensor(y, op="GET_ROWS", src=(src,), flags=G.FLAG_COMPUTE)
    assert g.compute([skipped, view, empty]) == (0, -1)
    assert bool((y == 7.0).all())
    assert g.compute([skipped, view, rows]) == (-3, 2)
    g.close()
