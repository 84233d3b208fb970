"""Llama-architecture decoder run op by op the way the reference's LNS backends
run a llama.cpp graph (SmolLM2-135M shape, random
weights): every ggml op reads F32, converts to LNS, computes and writes F32
(the op-boundary requantisation), the KV cache is F16, and the ops come in
llama.cpp's order for the LLaMA graph:

    x = get_rows(tok_embd, ids)                               (F32 copy)
    per layer:
      h = rms_norm(x) * attn_norm
      q, k, v = Wq h, Wk h, Wv h                              (mul_mat)
      q, k = rope(q), rope(k)                                 (mode NORM, base 1e5)
      K, V cache <- k, v                                      (F32 -> F16)
      kq = K^T q per head (GQA: q head i uses kv head i / 3)  (mul_mat, F16 K)
      p = soft_max_ext(kq, causal mask, 1/sqrt(64))
      o = Wo (V p)                                            (mul_mat, F16 V)
      x = x + o
      h = rms_norm(x) * ffn_norm
      x = x + W_down swiglu(W_gate h, W_up h)
    logits = tok_embd (rms_norm(x_last) * output_norm)        (tied output)

Ops carry llama.cpp-style tensor names (norm-<il>, Qcur/Kcur/Vcur-<il>,
kq-<il>, kq_soft_max-<il>, kqv-<il>, attn_out-<il> over kqv_out-<il>,
ffn_up/ffn_gate/ffn_down-<il>, result_output), which a summation policy
(lnsb200.policy, LNS16_SUM_POLICY) matches to pick each reduction's mode.

`forward` is written once over an ops object: GpuOps runs it through this
package's kernels (liblnsb200_<mode>.so); the CPU checker's ops object
(oracle/oracle_model.py, test infrastructure) runs the same graph through the
oracle.  Greedy decoding takes the
first largest logit (llama.cpp's greedy sampler).

Weights are drawn in a fixed order from numpy default_rng(seed) N(0, 0.02),
F32; the norm weights are 1.0.  The prompt is `prompt_len` ids from a separate
default_rng(seed).integers(0, vocab).
"""
import math

import numpy as np

SMOLLM2_135M = dict(n_layer=30, n_embd=576, n_head=9, n_head_kv=3, head_dim=64, n_ff=1536, vocab=49152,
                    rope_base=100000.0, eps=1e-5)


def init_weights(cfg, seed=2):
    """F32 weights as ggml holds them: a matrix of ne = (K, M) is M rows of K."""
    rng = np.random.default_rng(seed)
    E, F, V = cfg["n_embd"], cfg["n_ff"], cfg["vocab"]
    kv = cfg["n_head_kv"] * cfg["head_dim"]
    nrm = lambda *s: rng.normal(0.0, 0.02, s).astype(np.float32)
    w = {"tok_embd": nrm(V, E), "layers": []}
    for _ in range(cfg["n_layer"]):
        w["layers"].append({
            "attn_norm": np.ones(E, np.float32), "wq": nrm(E, E), "wk": nrm(kv, E), "wv": nrm(kv, E), "wo": nrm(E, E),
            "ffn_norm": np.ones(E, np.float32), "w_gate": nrm(F, E), "w_up": nrm(F, E), "w_down": nrm(E, F)})
    w["output_norm"] = np.ones(E, np.float32)
    return w


def prompt_ids(cfg, n, seed=2):
    return [int(v) for v in np.random.default_rng(seed).integers(0, cfg["vocab"], n)]


def rope_table(n_ctx, n_dims, base):
    """(cos, sin) per position and pair for positions 0 .. n_ctx-1, computed
    on the host in lns_rope's float recurrence (lns-backend/src/lns-ops.cpp:
    1231-1262) with the C library's cosf / sinf / powf; [n_ctx][n_dims/2][2]"""
    import ctypes
    libm = ctypes.CDLL("libm.so.6")
    for fn in ("cosf", "sinf"):
        getattr(libm, fn).restype = ctypes.c_float
        getattr(libm, fn).argtypes = [ctypes.c_float]
    libm.powf.restype = ctypes.c_float
    libm.powf.argtypes = [ctypes.c_float, ctypes.c_float]
    half = n_dims // 2
    ts = np.float32(libm.powf(float(np.float32(base)), float(np.float32(-2.0) / np.float32(n_dims))))
    out = np.empty((n_ctx, half, 2), np.float32)
    for p in range(n_ctx):
        t = np.float32(p)
        for j in range(half):
            out[p, j, 0] = libm.cosf(float(t))
            out[p, j, 1] = libm.sinf(float(t))
            t = np.float32(t * ts)
    return out


def forward(ops, cfg, ids, pos0):
    """logits (F32, [vocab]) of the last of `ids`, which sit at positions
    pos0 .. pos0 + len(ids) - 1; the KV cache holds positions < pos0."""
    if getattr(ops, "fused", False) and (ids.numel() if hasattr(ids, "numel") else len(ids)) == 1:
        return ops.forward_fused(cfg, ids, pos0)            # a decode step: the fused ops
    T, E = (ids.numel() if hasattr(ids, "numel") else len(ids)), cfg["n_embd"]
    H, HKV, D = cfg["n_head"], cfg["n_head_kv"], cfg["head_dim"]
    x = ops.embed(ids)                                              # [T][E]
    for il in range(cfg["n_layer"]):
        h = ops.mul(ops.rms_norm(x, cfg["eps"], "norm-%d" % il), ops.w(il, "attn_norm"))
        q, k, v = ops.linears(il, ("wq", "wk", "wv"), h,            # [T][H*D], [T][HKV*D] x 2
                              ("Qcur-%d" % il, "Kcur-%d" % il, "Vcur-%d" % il), "attn_norm-%d" % il)
        q = ops.rope(q, T, H, D, pos0)
        k = ops.rope(k, T, HKV, D, pos0)
        ops.kv_store(il, k, v, pos0, T)
        a = ops.attention(il, q, T, H, HKV, D, pos0)                # [T][H*D]
        x = ops.add(ops.linear(ops.w(il, "wo"), a, "attn_out-%d" % il, "kqv_out-%d" % il), x)
        h = ops.mul(ops.rms_norm(x, cfg["eps"], "norm-%d" % il), ops.w(il, "ffn_norm"))
        up, gate = ops.linears(il, ("w_up", "w_gate"), h, ("ffn_up-%d" % il, "ffn_gate-%d" % il), "ffn_norm-%d" % il)
        x = ops.add(ops.linear(ops.w(il, "w_down"), ops.swiglu(gate, up), "ffn_down-%d" % il, "ffn_swiglu-%d" % il), x)
    h = ops.mul(ops.rms_norm(ops.last_row(x), cfg["eps"], "norm"), ops.w(None, "output_norm"))
    return ops.linear(ops.w(None, "output"), h, "result_output", "result_norm")   # [1][vocab]


def generate(ops, cfg, prompt, n_gen):
    """prefill the prompt in one batch, then greedy-decode n_gen tokens"""
    logits = forward(ops, cfg, prompt, 0)
    out = []
    pos = len(prompt)
    for _ in range(n_gen):
        tok = ops.argmax(logits)
        out.append(tok)
        if len(out) == n_gen:
            break
        logits = forward(ops, cfg, [tok], pos)
        pos += 1
    return out


class GpuOps:
    """The graph's ops through liblnsb200_<mode>.so on one CUDA device (torch
    for memory and the non-arithmetic reshapes)."""

    def __init__(self, cfg, weights, mode="sum32", n_ctx=256, stream=None, fmt=16, policy=None):
        import torch
        import lnsb200
        from .policy import SumPolicy
        self.torch, self.cfg, self.n_ctx = torch, cfg, n_ctx
        self.fmt = fmt
        self.cdt = torch.int16 if fmt == 16 else torch.int32             # LNS code storage
        self.ks = lnsb200.KernelSet(fmt, mode)
        self.ks.upload_tables()
        # xlns16 only: a summation mode per op (the default: `mode`)
        self.policy = SumPolicy(policy, mode) if fmt == 16 and policy else None
        self.kss = {mode: self.ks}
        self.weights = weights
        self.split_w = {}
        self.fuse_attn = True           # decode steps (T = 1) through lnsb_attn_decode
        # the whole step through the fused ops (norm block, rope + KV store, attention,
        # glu + to_lns) when one summation mode serves every op
        self.fused = self.policy is None
        self.stream = stream
        self.dev = torch.device("cuda", torch.cuda.current_device())
        E = cfg["n_embd"]
        kvd = cfg["n_head_kv"] * cfg["head_dim"]
        self.tok_embd = torch.from_numpy(weights["tok_embd"]).to(self.dev)
        self.lw = []
        for L in weights["layers"]:
            # q/k/v and up/gate share their input: one mul_mat over the stacked
            # rows computes the same chains (each output is its own reduction)
            d = {"qkv": self._weight(np.concatenate([L["wq"], L["wk"], L["wv"]])),
                 "upgate": self._weight(np.concatenate([L["w_up"], L["w_gate"]])),
                 "split": {("wq", "wk", "wv"): [L["wq"].shape[0], L["wk"].shape[0], L["wv"].shape[0]],
                           ("w_up", "w_gate"): [L["w_up"].shape[0], L["w_gate"].shape[0]]}}
            for name in ("wo", "w_down"):
                d[name] = self._weight(L[name])
            for name in ("attn_norm", "ffn_norm"):
                d[name] = torch.from_numpy(L[name]).to(self.dev)
            self.lw.append(d)
        self.gw = {"output_norm": torch.from_numpy(weights["output_norm"]).to(self.dev),
                   "output": self._weight(weights["tok_embd"])}
        self.kc = [torch.empty((n_ctx, kvd), dtype=torch.int16, device=self.dev) for _ in weights["layers"]]
        self.vc = [torch.empty((n_ctx, kvd), dtype=torch.int16, device=self.dev) for _ in weights["layers"]]
        self.rope_cs = torch.from_numpy(rope_table(n_ctx, cfg["head_dim"], cfg["rope_base"])).to(self.dev)
        neg = np.full((n_ctx, n_ctx), -np.inf, np.float32)
        self.mask_full = torch.from_numpy(np.triu(neg, 1)).to(self.dev)     # row q: 0 for k <= q
        self.launches = 0

    # weights: F32 rows [M][K] -> xlns16 codes k-major [K][M], once (the weight cache)
    def _weight(self, rows):
        torch = self.torch
        M, K = rows.shape
        src = torch.from_numpy(np.ascontiguousarray(rows)).to(self.dev)
        dst = torch.empty(K * M, dtype=self.cdt, device=self.dev)
        self.ks.to_lns_transposed(src, dst, M, K, M)
        torch.cuda.synchronize()
        return (dst, K, M)

    def w(self, il, name):
        return self.gw[name] if il is None else self.lw[il][name]

    def _f32(self, *shape):
        return self.torch.empty(shape, dtype=self.torch.float32, device=self.dev)

    def embed(self, ids):
        if isinstance(ids, self.torch.Tensor):                          # token ids already on the device
            return self.tok_embd.index_select(0, ids.view(-1)).contiguous()
        return self.tok_embd[self.torch.tensor(ids, device=self.dev)].contiguous()

    def ks_for(self, op, name, src1=None):
        """the kernel set of the op's summation mode"""
        if self.policy is None:
            return self.ks
        mode = self.policy.mode_for(op, name, src1)
        if mode not in self.kss:
            import lnsb200
            self.kss[mode] = lnsb200.KernelSet(self.fmt, mode)
            self.kss[mode].upload_tables()
        return self.kss[mode]

    def rms_norm(self, x, eps, name=None):
        out = self._f32(*x.shape)
        self.ks_for("RMS_NORM", name).rms_norm(x, out, x.shape[-1], x.numel() // x.shape[-1], eps, stream=self.stream)
        self.launches += 1
        return out

    def mul(self, x, wv):
        out = self._f32(*x.shape)
        self.ks.binary("mul", x, (x.shape[-1], x.numel() // x.shape[-1]), wv, (wv.numel(),), out, stream=self.stream)
        self.launches += 1
        return out

    def add(self, a, b):
        out = self._f32(*a.shape)
        self.ks.binary("add", a, (a.shape[-1], a.numel() // a.shape[-1]), b, (b.shape[-1], b.numel() // b.shape[-1]),
                       out, stream=self.stream)
        self.launches += 1
        return out

    def linear(self, wt, x, name=None, src1=None):
        codes, K, M = wt
        N = x.numel() // K
        xl = self.torch.empty(N * K, dtype=self.cdt, device=self.dev)
        self.ks.to_lns(x, xl, stream=self.stream)
        out = self._f32(N, M)
        self.ks_for("MUL_MAT", name, src1).mul_mat(codes, xl, out, K, M, N, stream=self.stream)
        self.launches += 2
        return out

    def linears(self, il, names, x, tnames=None, src1=None):
        tnames = tnames or (None,) * len(names)
        kss = {id(self.ks_for("MUL_MAT", t, src1)) for t in tnames}
        if len(kss) > 1:                                # the policy splits the group: one mul_mat per weight
            outs = []
            for n, t in zip(names, tnames):
                if (il, n) not in self.split_w:
                    self.split_w[(il, n)] = self._weight(self.weights["layers"][il][n])
                outs.append(self.linear(self.split_w[(il, n)], x, t, src1))
            return outs
        key = "qkv" if names[0] == "wq" else "upgate"
        y = self.linear(self.lw[il][key], x, tnames[0], src1)
        outs, c = [], 0
        for m in self.lw[il]["split"][tuple(names)]:
            outs.append(y[:, c:c + m].contiguous())
            c += m
        return outs

    def rope(self, x, T, nh, hd, pos0):
        out = self._f32(T, nh * hd)
        self.ks.rope(x, (hd, nh, T, 1), self.rope_cs[pos0:pos0 + T], hd, out, stream=self.stream)
        self.launches += 1
        return out

    def kv_store(self, il, k, v, pos0, T):
        n = k.numel()
        self.ks.f32_to_f16(k, self.kc[il][pos0:pos0 + T], n, stream=self.stream)
        self.ks.f32_to_f16(v, self.vc[il][pos0:pos0 + T], n, stream=self.stream)
        self.launches += 2

    def attention(self, il, q, T, H, HKV, D, pos0):
        torch, ks = self.torch, self.ks
        nkv = pos0 + T
        if T == 1 and self.fuse_attn and nkv <= ks.attn_decode_max_keys(D) and all(self.ks_for(op, n) is ks for op, n in (
                ("MUL_MAT", "kq-%d" % il), ("SOFT_MAX", "kq_soft_max-%d" % il), ("MUL_MAT", "kqv-%d" % il))):
            # one decode step: the fused kernel runs the same ops with the same conversions
            o = self._f32(1, H * D)
            ks.attn_decode(q, self.kc[il], self.vc[il], HKV * D, nkv, H, HKV, D, 1.0 / math.sqrt(D), o,
                           stream=self.stream)
            self.launches += 1
            return o
        # K and V of the cache, F16 -> F32 -> xlns16 codes, laid out as mul_mat weights per kv head:
        # K: [h][dim][token] (reduce over dim), V: [h][token][dim] (reduce over tokens)
        kf = self._f32(nkv, HKV * D)
        vf = self._f32(nkv, HKV * D)
        ks.f16_to_f32(self.kc[il][:nkv], kf, kf.numel(), stream=self.stream)
        ks.f16_to_f32(self.vc[il][:nkv], vf, vf.numel(), stream=self.stream)
        kh = kf.view(nkv, HKV, D).permute(1, 0, 2).contiguous()          # [h][token][dim] F32
        vh = vf.view(nkv, HKV, D).permute(1, 0, 2).contiguous()
        kl = torch.empty(HKV * D * nkv, dtype=self.cdt, device=self.dev)
        vl = torch.empty(HKV * nkv * D, dtype=self.cdt, device=self.dev)
        for h in range(HKV):
            ks.to_lns_transposed(kh[h], kl[h * D * nkv:(h + 1) * D * nkv], nkv, D, nkv, stream=self.stream)
        ks.to_lns(vh, vl, stream=self.stream)
        # kq[h][t][k] = sum_d K[k][d] q[t][d], q head h on kv head h / (H / HKV)
        qh = q.view(T, H, D).permute(1, 0, 2).contiguous()                # [h][t][dim]
        ql = torch.empty(qh.numel(), dtype=self.cdt, device=self.dev)
        ks.to_lns(qh, ql, stream=self.stream)
        kq = self._f32(H, T, nkv)
        self.ks_for("MUL_MAT", "kq-%d" % il).mul_mat(kl, ql, kq, D, nkv, T, (HKV, 1, H, 1), stream=self.stream)
        # causal mask rows pos0 .. pos0+T-1, scale 1/sqrt(head_dim)
        mask = self.mask_full[pos0:pos0 + T, :nkv].contiguous()
        p = self._f32(H, T, nkv)
        work = torch.empty(p.numel(), dtype=self.cdt, device=self.dev)
        self.ks_for("SOFT_MAX", "kq_soft_max-%d" % il).soft_max(kq, (nkv, T, H, 1), p, work, mask, (nkv, T, 1, 1),
                                                               1.0 / math.sqrt(D), stream=self.stream)
        # o[h][t][d] = sum_k V[k][d] p[h][t][k]
        pl = torch.empty(p.numel(), dtype=self.cdt, device=self.dev)
        ks.to_lns(p, pl, stream=self.stream)
        o = self._f32(H, T, D)
        self.ks_for("MUL_MAT", "kqv-%d" % il).mul_mat(vl, pl, o, nkv, D, T, (HKV, 1, H, 1), stream=self.stream)
        self.launches += 9 + HKV
        return o.permute(1, 0, 2).contiguous().view(T, H * D)

    def swiglu(self, gate, up):
        out = self._f32(*gate.shape)
        nc = gate.shape[-1]
        self.ks.glu(gate, up, nc, nc, out, nc, gate.numel() // nc, stream=self.stream)
        self.launches += 1
        return out

    def last_row(self, x):
        return x[-1:].contiguous()

    def argmax(self, logits):
        return int(self.torch.argmax(logits.view(-1)).item())

    def _codes(self, *shape):
        return self.torch.empty(shape, dtype=self.cdt, device=self.dev)

    def _mv(self, wt, xc, N):
        codes, K, M = wt
        out = self._f32(N, M)
        self.ks.mul_mat(codes, xc, out, K, M, N, stream=self.stream)
        return out

    def forward_fused(self, cfg, ids, pos0):
        """forward() with the fused steps: per layer a norm block (residual add,
        rms_norm, weight, to_lns), the q/k/v mat-vec, rope + KV store, the
        attention (fused for a decode step), wo, a norm block, up/gate, glu +
        to_lns, down -- nine launches, the same bits as the op-by-op graph"""
        ks, torch = self.ks, self.torch
        T = ids.numel() if hasattr(ids, "numel") else len(ids)
        E, H, HKV, D, F = cfg["n_embd"], cfg["n_head"], cfg["n_head_kv"], cfg["head_dim"], cfg["n_ff"]
        eps, kvd, nkv, s = cfg["eps"], HKV * D, pos0 + T, self.stream
        x = self.embed(ids)                                          # [T][E]
        res = None                                                   # the pending residual add (a, x)
        for il in range(cfg["n_layer"]):
            lw = self.lw[il]
            hc = self._codes(T * E)
            if res is None:
                ks.norm_block(x, hc, E, T, eps, weight=lw["attn_norm"], stream=s)
            else:
                xn = self._f32(T, E)
                ks.norm_block(res[0], hc, E, T, eps, residual=res[1], x_out=xn, weight=lw["attn_norm"], stream=s)
                x = xn
            qkv = self._mv(lw["qkv"], hc, T)                         # [T][(H + 2 HKV) D]
            q = self._f32(T, H * D)
            ks.rope_qkv(qkv, (H + 2 * HKV) * D, self.rope_cs[pos0:pos0 + T], D, H, HKV, D, T, q,
                        self.kc[il][pos0:pos0 + T], self.vc[il][pos0:pos0 + T], kvd, stream=s)
            ac = self._codes(T * H * D)
            if T == 1 and self.fuse_attn and nkv <= ks.attn_decode_max_keys(D):
                ks.attn_decode(q, self.kc[il], self.vc[il], kvd, nkv, H, HKV, D, 1.0 / math.sqrt(D), None,
                               stream=s, dst_lns=ac)
            else:
                ks.to_lns(self.attention(il, q, T, H, HKV, D, pos0), ac, stream=s)
            wo = self._mv(lw["wo"], ac, T)
            hc = self._codes(T * E)
            xn = self._f32(T, E)
            ks.norm_block(wo, hc, E, T, eps, residual=x, x_out=xn, weight=lw["ffn_norm"], stream=s)
            x = xn
            ug = self._mv(lw["upgate"], hc, T)                       # [T][up | gate]
            sc = self._codes(T * F)
            ks.glu_lns(ug[:, F:], ug, 2 * F, 2 * F, sc, F, T, stream=s)
            res = (self._mv(lw["w_down"], sc, T), x)
        hc = self._codes(E)
        ks.norm_block(res[0][T - 1:], hc, E, 1, eps, residual=res[1][T - 1:], weight=self.gw["output_norm"], stream=s)
        self.launches += 9 * cfg["n_layer"] + 2
        return self._mv(self.gw["output"], hc, 1)                    # [1][vocab]


class GraphDecoder:
    """Greedy decode with one CUDA graph per position: the step at position
    pos (embedding of the current token, the 30 layers, the output matmul,
    argmax into the device token, and the token's copy to pinned host memory)
    is captured once and replayed, so a decode step costs no host work.  The
    kernels and their order are those of the eager path."""

    def __init__(self, ops, cfg):
        import torch
        self.torch, self.ops, self.cfg = torch, ops, cfg
        self.tok = torch.zeros(1, dtype=torch.int64, device=ops.dev)
        self.host = torch.zeros(ops.n_ctx, dtype=torch.int64).pin_memory()
        self.graphs = {}
        self.logits = {}                 # each position's logits: the graph's own output buffer

    def capture(self, pos):
        torch = self.torch
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            logits = forward(self.ops, self.cfg, self.tok, pos)
            self.tok.copy_(torch.argmax(logits.view(-1)).view(1))
            self.host[pos:pos + 1].copy_(self.tok, non_blocking=True)
        self.graphs[pos] = g
        self.logits[pos] = logits

    def prepare(self, pos_from, pos_to):
        """capture the steps at positions pos_from .. pos_to - 1 (after one eager
        step has set every kernel's launch attributes)"""
        # one eager step first, at the last position (its cache slot is written
        # again by that position's own step before anything reads it), so no
        # kernel's first-use setup falls inside a capture
        forward(self.ops, self.cfg, self.tok, pos_to - 1)
        self.torch.cuda.synchronize()
        for p in range(pos_from, pos_to):
            if p not in self.graphs:
                self.capture(p)

    def step(self, pos, token=None):
        """replays position pos (after setting the current token, if given) and
        returns that step's logits (device tensor, valid until pos replays again)"""
        if token is not None:
            self.tok.fill_(token)
        self.graphs[pos].replay()
        return self.logits[pos]

    def decode(self, first_token, pos_from, n):
        """n tokens: first_token is the one the prefill produced (at pos_from)"""
        self.tok.fill_(first_token)
        for p in range(pos_from, pos_from + n):
            self.graphs[p].replay()
        self.torch.cuda.current_stream().synchronize()
        return [int(v) for v in self.host[pos_from:pos_from + n]]
