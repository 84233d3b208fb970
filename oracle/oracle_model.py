"""The LLaMA graph of lnsb200.model on the CPU through the oracle.

TEST INFRASTRUCTURE ONLY: the checker of lnsb200.model.GpuOps (the tests and
bench.py's CPU-baseline leg use it; the product package never imports it).
`lnsb200.model.forward` runs over either ops object, so both run the same
graph op by op.
"""
import math
import os
import sys

import numpy as np

_PKG = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "xlns-ggml-backend_b200")
if _PKG not in sys.path:
    sys.path.insert(0, _PKG)

from lnsb200.model import rope_table  # noqa: E402


class OracleOps:
    """The same ops on the CPU through the oracle (test infrastructure only:
    the checker of GpuOps)."""

    def __init__(self, cfg, weights, mode="sum32", n_ctx=256, nthreads=8, fmt=16, policy=None):
        import oracle
        from lnsb200.policy import SumPolicy
        self.o, self.cfg, self.mode, self.nt, self.fmt = oracle, cfg, mode, nthreads, fmt
        self.policy = SumPolicy(policy, mode) if fmt == 16 and policy else None
        o = oracle
        if fmt == 16:
            self.to_c, self.to_f, self.mask_c = o.from_f32_16, o.to_f32_16, o.mask16
            self.mm = lambda md, w, x, **kw: o.mul_mat16(md, w, x, **kw)
            self.rms = lambda md, c, nc, nr, eps: o.rms_norm16(md, c, nc, nr, eps, nthreads=nthreads)
            self.smax = lambda md, c, shp, m, mshp, sc: o.soft_max16(md, c, shp, m, mshp, sc, nthreads=nthreads)
        else:
            self.to_c, self.to_f, self.mask_c = o.from_f32_32, o.to_f32_32, o.mask32
            self.mm = lambda md, w, x, **kw: o.mul_mat32(w, x, **kw)
            self.rms = lambda md, c, nc, nr, eps: o.rms_norm32(c, nc, nr, eps, nthreads=nthreads)
            self.smax = lambda md, c, shp, m, mshp, sc: o.soft_max32(c, shp, m, mshp, sc, nthreads=nthreads)
        self.weights = weights
        self.wc = {}
        kvd = cfg["n_head_kv"] * cfg["head_dim"]
        self.kc = [np.zeros((n_ctx, kvd), np.float16) for _ in weights["layers"]]
        self.vc = [np.zeros((n_ctx, kvd), np.float16) for _ in weights["layers"]]
        self.rope_cs = rope_table(n_ctx, cfg["head_dim"], cfg["rope_base"])

    def w(self, il, name):
        key = (il, name)
        if key not in self.wc:
            if il is None:
                v = self.weights["tok_embd"] if name == "output" else self.weights[name]
            else:
                v = self.weights["layers"][il][name]
            if v.ndim == 2:
                v = self.to_c(v)                               # weight codes, rows [M][K]
            self.wc[key] = v
        return self.wc[key]

    def embed(self, ids):
        return self.weights["tok_embd"][ids].copy()

    def mode_for(self, op, name, src1=None):
        return self.policy.mode_for(op, name, src1) if self.policy is not None else self.mode

    def rms_norm(self, x, eps, name=None):
        c = self.to_c(x)
        r = self.rms(self.mode_for("RMS_NORM", name), c.ravel(), x.shape[-1], x.size // x.shape[-1], eps)
        return self.to_f(r).reshape(x.shape)

    def mul(self, x, wv):
        return self.o.binary16("mul", x, wv.reshape(1, -1), fmt=self.fmt)

    def add(self, a, b):
        return self.o.binary16("add", a, b, fmt=self.fmt)

    def linear(self, w, x, name=None, src1=None):
        xc = self.to_c(x.reshape(-1, w.shape[1]))
        return self.to_f(self.mm(self.mode_for("MUL_MAT", name, src1), w, xc, nthreads=self.nt)).reshape(-1, w.shape[0])

    def linears(self, il, names, x, tnames=None, src1=None):
        tnames = tnames or (None,) * len(names)
        return [self.linear(self.w(il, n), x, t, src1) for n, t in zip(names, tnames)]

    def rope(self, x, T, nh, hd, pos0):
        return self.o.rope16(x.reshape(1, T, nh, hd), self.rope_cs[pos0:pos0 + T], hd, fmt=self.fmt).reshape(T, nh * hd)

    def kv_store(self, il, k, v, pos0, T):
        self.kc[il][pos0:pos0 + T] = k.astype(np.float16)
        self.vc[il][pos0:pos0 + T] = v.astype(np.float16)

    def attention(self, il, q, T, H, HKV, D, pos0):
        o = self.o
        nkv = pos0 + T
        kf = self.kc[il][:nkv].astype(np.float32).reshape(nkv, HKV, D)
        vf = self.vc[il][:nkv].astype(np.float32).reshape(nkv, HKV, D)
        kw = self.to_c(np.ascontiguousarray(kf.transpose(1, 0, 2)))            # [h][token][dim]: rows M=token, K=dim
        vw = self.to_c(np.ascontiguousarray(vf.transpose(1, 2, 0)))            # [h][dim][token]: rows M=dim, K=token
        qc = self.to_c(np.ascontiguousarray(q.reshape(T, H, D).transpose(1, 0, 2)))
        kq = self.to_f(self.mm(self.mode_for("MUL_MAT", "kq-%d" % il), kw.reshape(1, HKV, nkv, D),
                               qc.reshape(1, H, T, D), slices=(HKV, 1, H, 1), nthreads=self.nt)).reshape(H, T, nkv)
        m = np.triu(np.full((T + pos0, T + pos0), -np.inf, np.float32), 1)[pos0:pos0 + T, :nkv]
        sc = int(self.to_c(np.array([1.0 / math.sqrt(D)], np.float32))[0])
        p = self.to_f(self.smax(self.mode_for("SOFT_MAX", "kq_soft_max-%d" % il), self.to_c(kq).ravel(), (nkv, T, H, 1),
                                self.mask_c(m).ravel(), (nkv, T, 1, 1), sc)).reshape(H, T, nkv)
        out = self.to_f(self.mm(self.mode_for("MUL_MAT", "kqv-%d" % il), vw.reshape(1, HKV, D, nkv),
                                self.to_c(p).reshape(1, H, T, nkv), slices=(HKV, 1, H, 1), nthreads=self.nt)).reshape(H, T, D)
        return np.ascontiguousarray(out.transpose(1, 0, 2)).reshape(T, H * D)

    def swiglu(self, gate, up):
        return self.o.swiglu16(gate, up, fmt=self.fmt)

    def last_row(self, x):
        return x[-1:].copy()

    def argmax(self, logits):
        return int(np.argmax(logits.ravel()))
