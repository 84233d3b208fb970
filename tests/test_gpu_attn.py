"""The fused decode attention (lnsb_attn_decode) against the same step run op
by op (F16 -> F32, to_lns, mul_mat kq, soft_max, to_lns, mul_mat kqv) and
against the CPU oracle's graph, bit for bit, in every summation-mode build
and in xlns32 (Monte chains included: the fused kernel starts each chain
where the unfused calls start it)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

CFG = dict(n_layer=1, n_embd=576, n_head=9, n_head_kv=3, head_dim=64, n_ff=64, vocab=64, rope_base=100000.0, eps=1e-5)


def caches(rng, n_ctx, kvd):
    k = rng.normal(0, 1.0, (n_ctx, kvd)).astype(np.float16)
    v = rng.normal(0, 1.0, (n_ctx, kvd)).astype(np.float16)
    return k, v


@pytest.mark.parametrize("fmt,mode", [(16, "base"), (16, "monte"), (16, "monte_bylpvip"), (16, "lpvip"), (16, "sum32"),
                                      (32, "base")])
@pytest.mark.parametrize("nkv", [1, 37, 300])
def test_attn_decode_matches_unfused_and_oracle(fmt, mode, nkv):
    from lnsb200 import model
    from oracle_model import OracleOps
    rng = np.random.default_rng(nkv + fmt)
    H, HKV, D = CFG["n_head"], CFG["n_head_kv"], CFG["head_dim"]
    w = model.init_weights(CFG, seed=1)
    g = model.GpuOps(CFG, w, mode=mode, n_ctx=320, fmt=fmt)
    k, v = caches(rng, 320, HKV * D)
    g.kc[0].copy_(torch.from_numpy(k.view(np.int16)).cuda())
    g.vc[0].copy_(torch.from_numpy(v.view(np.int16)).cuda())
    q = torch.from_numpy(rng.normal(0, 2.0, (1, H * D)).astype(np.float32)).cuda()
    fused = g.attention(0, q, 1, H, HKV, D, nkv - 1).cpu().numpy()
    g.fuse_attn = False
    plain = g.attention(0, q, 1, H, HKV, D, nkv - 1).cpu().numpy()
    assert np.array_equal(fused.view(np.uint32), plain.view(np.uint32))
    o = OracleOps(CFG, w, mode=mode, n_ctx=320, fmt=fmt)
    o.kc[0][:] = k
    o.vc[0][:] = v
    want = o.attention(0, q.cpu().numpy(), 1, H, HKV, D, nkv - 1)
    assert np.array_equal(fused.ravel().view(np.uint32), want.ravel().view(np.uint32))


def test_attn_decode_too_long_and_invalid():
    import lnsb200
    ks = lnsb200.KernelSet(16, "sum32")
    ks.upload_tables()
    z16 = torch.zeros(64, dtype=torch.int16, device="cuda")
    zf = torch.zeros(64, dtype=torch.float32, device="cuda")
    mk = ks.attn_decode_max_keys(64)
    assert 2000 < mk < 8000
    with pytest.raises(lnsb200.LnsbError):
        ks.attn_decode(zf, z16, z16, 64, mk + 1, 1, 1, 64, 0.125, zf)     # too many keys for shared memory
    with pytest.raises(lnsb200.LnsbError):
        ks.attn_decode(zf, z16, z16, 64, 4, 9, 2, 64, 0.125, zf)           # 9 heads over 2 kv heads
