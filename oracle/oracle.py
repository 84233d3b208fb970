"""ctypes access to the CPU oracle (oracle/_build/liblns_oracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg, as the checker.  The product never imports it.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD = os.path.join(HERE, "_build")
SO = os.path.join(BUILD, "liblns_oracle.so")
PINCHECK = os.path.join(BUILD, "pincheck")

MODE = {"base": 0, "monte": 1, "monte_bylpvip": 2, "lpvip": 3, "sum32": 4}

_lib = None


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(SO):
            build()
        L = ctypes.CDLL(SO)
        u16p = np.ctypeslib.ndpointer(np.uint16, flags="C")
        u32p = np.ctypeslib.ndpointer(np.uint32, flags="C")
        i32p = np.ctypeslib.ndpointer(np.int32, flags="C")
        f32p = np.ctypeslib.ndpointer(np.float32, flags="C")
        i64 = ctypes.c_int64
        i64a = ctypes.POINTER(ctypes.c_int64)
        sig = {
            "orc_init": (ctypes.c_int, []),
            "orc16_from_f32": (ctypes.c_uint16, [ctypes.c_float]),
            "orc16_to_f32": (ctypes.c_float, [ctypes.c_uint16]),
            "orc16_add": (ctypes.c_uint16, [ctypes.c_uint16, ctypes.c_uint16]),
            "orc16_mul": (ctypes.c_uint16, [ctypes.c_uint16, ctypes.c_uint16]),
            "orc32_add": (ctypes.c_uint32, [ctypes.c_uint32, ctypes.c_uint32]),
            "orc32_from_f32": (ctypes.c_uint32, [ctypes.c_float]),
            "orc_lfsr_step": (ctypes.c_uint16, [ctypes.c_uint16]),
            "orc_lfsr_jump": (ctypes.c_uint16, [ctypes.c_uint16, ctypes.c_uint64]),
            "orc_mul_mat_draws": (ctypes.c_uint64, [ctypes.c_int, i64, i64, i64, i64, i64]),
            "orc_soft_max_draws": (ctypes.c_uint64, [ctypes.c_int, i64, i64]),
            "orc_rms_norm_draws": (ctypes.c_uint64, [ctypes.c_int, i64, i64]),
            "orc16_mul_mat": (None, [ctypes.c_int, u16p, u16p, u16p, i64, i64, i64, i64, i64, i64, i64,
                                     ctypes.c_uint16, ctypes.c_int]),
            "orc32_mul_mat": (None, [u32p, u32p, u32p, i64, i64, i64, i64, i64, i64, i64, ctypes.c_int]),
            "orc16_mul_mat_id": (i64, [ctypes.c_int, u16p, u16p, i32p, u16p, i64, i64, i64, i64, i64, i64, i64,
                                       ctypes.c_uint16, ctypes.c_int]),
            "orc32_mul_mat_id": (i64, [u32p, u32p, i32p, u32p, i64, i64, i64, i64, i64, i64, i64, ctypes.c_int]),
            "orc16_soft_max": (None, [ctypes.c_int, u16p, i64a, ctypes.c_void_p, i64a, ctypes.c_uint16, u16p,
                                      ctypes.c_uint16, ctypes.c_int]),
            "orc32_soft_max": (None, [u32p, i64a, ctypes.c_void_p, i64a, ctypes.c_uint32, u32p, ctypes.c_int]),
            "orc16_rms_norm": (None, [ctypes.c_int, u16p, u16p, i64, i64, ctypes.c_float, ctypes.c_uint16, ctypes.c_int]),
            "orc32_rms_norm": (None, [u32p, u32p, i64, i64, ctypes.c_float, ctypes.c_int]),
            "orc16_mask_from_f32": (ctypes.c_uint16, [ctypes.c_float]),
            "orc32_mask_from_f32": (ctypes.c_uint32, [ctypes.c_float]),
            "orc16_from_f32_n": (None, [f32p, u16p, i64]),
            "orc16_to_f32_n": (None, [u16p, f32p, i64]),
            "orc32_from_f32_n": (None, [f32p, u32p, i64]),
            "orc32_to_f32_n": (None, [u32p, f32p, i64]),
            "orc16_silu": (ctypes.c_uint16, [ctypes.c_uint16]),
            "orc16_binary_f32": (None, [ctypes.c_int, f32p, i64a, f32p, i64a, f32p]),
            "orc16_scale_f32": (None, [f32p, f32p, i64, ctypes.c_float, ctypes.c_float]),
            "orc16_unary_f32": (None, [ctypes.c_int, f32p, f32p, i64]),
            "orc32_unary_f32": (None, [ctypes.c_int, f32p, f32p, i64]),
            "orc16_swiglu_f32": (None, [f32p, f32p, i64, i64, f32p, i64, i64]),
            "orc16_rope_f32": (None, [f32p, i64a, f32p, ctypes.c_int, ctypes.c_int, f32p]),
            "orc32_binary_f32": (None, [ctypes.c_int, f32p, i64a, f32p, i64a, f32p]),
            "orc32_scale_f32": (None, [f32p, f32p, i64, ctypes.c_float, ctypes.c_float]),
            "orc32_swiglu_f32": (None, [f32p, f32p, i64, i64, f32p, i64, i64]),
            "orc16_geglu_f32": (None, [f32p, f32p, i64, i64, f32p, i64, i64]),
            "orc32_geglu_f32": (None, [f32p, f32p, i64, i64, f32p, i64, i64]),
            "orc32_rope_f32": (None, [f32p, i64a, f32p, ctypes.c_int, ctypes.c_int, f32p]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        if L.orc_init() != 0:
            raise RuntimeError("oracle table construction failed")
        _lib = L
    return _lib


BINARY = {"add": 0, "mul": 1, "div": 2}
UNARY = {"silu": 0, "gelu": 1, "relu": 2, "tanh": 3}


def binary16(op, a, b, fmt=16):
    """a op b at the F32 op boundary, b repeated to a's shape (numpy, innermost last)."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    out = np.empty_like(a)
    fn = lib().orc16_binary_f32 if fmt == 16 else lib().orc32_binary_f32
    fn(BINARY[op], a.ravel(), _ne(a.shape[::-1]), b.ravel(), _ne(b.shape[::-1]), out.ravel())
    return out


def scale16(src, s, b=0.0, fmt=16):
    src = np.ascontiguousarray(src, np.float32)
    out = np.empty_like(src)
    (lib().orc16_scale_f32 if fmt == 16 else lib().orc32_scale_f32)(src.ravel(), out.ravel(), src.size, s, b)
    return out


def unary16(op, src, fmt=16):
    src = np.ascontiguousarray(src, np.float32)
    out = np.empty_like(src)
    (lib().orc16_unary_f32 if fmt == 16 else lib().orc32_unary_f32)(UNARY[op], src.ravel(), out.ravel(), src.size)
    return out


def swiglu16(gate, up, fmt=16, op="swiglu"):
    """act(gate) * up, rows of gate.shape[-1]; act = silu (swiglu) or gelu (geglu)"""
    gate = np.ascontiguousarray(gate, np.float32)
    up = np.ascontiguousarray(up, np.float32)
    nc = gate.shape[-1]
    out = np.empty_like(gate)
    fn = {("swiglu", 16): lib().orc16_swiglu_f32, ("swiglu", 32): lib().orc32_swiglu_f32,
          ("geglu", 16): lib().orc16_geglu_f32, ("geglu", 32): lib().orc32_geglu_f32}[(op, fmt)]
    fn(gate.ravel(), up.ravel(), nc, nc, out.ravel(), nc, gate.size // nc)
    return out


def rope16(src, cos_sin, n_dims, neox=False, fmt=16):
    """src [ne3][ne2][ne1][ne0] (numpy order), cos_sin [ne2][n_dims/2][2]"""
    src = np.ascontiguousarray(src, np.float32)
    cs = np.ascontiguousarray(cos_sin, np.float32)
    out = np.empty_like(src)
    (lib().orc16_rope_f32 if fmt == 16 else lib().orc32_rope_f32)(src.ravel(), _ne(src.shape[::-1]), cs.ravel(), n_dims,
                                                                   1 if neox else 0, out.ravel())
    return out


def rope_cos_sin(pos, n_dims, freq_base):
    """(cos, sin) per position and rotated pair in the float recurrence of
    lns_rope (lns-backend/src/lns-ops.cpp:1231-1262), with the C library's
    float functions: theta_scale = powf(base, -2/n_dims), t = pos,
    cos_sin = (cosf(t), sinf(t)), t *= theta_scale per pair."""
    libm = ctypes.CDLL("libm.so.6")
    for fn in ("cosf", "sinf"):
        getattr(libm, fn).restype = ctypes.c_float
        getattr(libm, fn).argtypes = [ctypes.c_float]
    libm.powf.restype = ctypes.c_float
    libm.powf.argtypes = [ctypes.c_float, ctypes.c_float]
    half = n_dims // 2
    ts = np.float32(libm.powf(float(np.float32(freq_base)), float(np.float32(-2.0) / np.float32(n_dims))))
    out = np.empty((len(pos), half, 2), np.float32)
    for i, p in enumerate(pos):
        t = np.float32(p)
        for j in range(half):
            out[i, j, 0] = libm.cosf(float(t))
            out[i, j, 1] = libm.sinf(float(t))
            t = np.float32(t * ts)
    return out


def _ne(shape):
    return (ctypes.c_int64 * 4)(*(list(shape) + [1] * (4 - len(shape))))


def from_f32_16(a):
    a = np.ascontiguousarray(a, np.float32)
    out = np.empty(a.shape, np.uint16)
    lib().orc16_from_f32_n(a.ravel(), out.ravel(), a.size)
    return out


def to_f32_16(c):
    c = np.ascontiguousarray(c, np.uint16)
    out = np.empty(c.shape, np.float32)
    lib().orc16_to_f32_n(c.ravel(), out.ravel(), c.size)
    return out


def from_f32_32(a):
    a = np.ascontiguousarray(a, np.float32)
    out = np.empty(a.shape, np.uint32)
    lib().orc32_from_f32_n(a.ravel(), out.ravel(), a.size)
    return out


def to_f32_32(c):
    c = np.ascontiguousarray(c, np.uint32)
    out = np.empty(c.shape, np.float32)
    lib().orc32_to_f32_n(c.ravel(), out.ravel(), c.size)
    return out


def mul_mat16(mode, w_rows, x, slices=(1, 1, 1, 1), seed=7, nthreads=1):
    """w_rows: codes [ne03][ne02][M][K] (weight rows), x: codes [ne13][ne12][N][K];
    returns codes [ne13][ne12][N][M]."""
    ne02, ne03, ne12, ne13 = slices
    M, K = w_rows.shape[-2], w_rows.shape[-1]
    N = x.shape[-2]
    w = np.ascontiguousarray(w_rows, np.uint16).reshape(-1)
    xx = np.ascontiguousarray(x, np.uint16).reshape(-1)
    out = np.empty(ne12 * ne13 * N * M, np.uint16)
    lib().orc16_mul_mat(MODE[mode], w, xx, out, K, M, N, ne02, ne03, ne12, ne13, seed, nthreads)
    return out.reshape(ne13, ne12, N, M) if (ne12 * ne13) > 1 else out.reshape(N, M)


def mul_mat32(w_rows, x, slices=(1, 1, 1, 1), nthreads=1):
    ne02, ne03, ne12, ne13 = slices
    M, K = w_rows.shape[-2], w_rows.shape[-1]
    N = x.shape[-2]
    w = np.ascontiguousarray(w_rows, np.uint32).reshape(-1)
    xx = np.ascontiguousarray(x, np.uint32).reshape(-1)
    out = np.empty(ne12 * ne13 * N * M, np.uint32)
    lib().orc32_mul_mat(w, xx, out, K, M, N, ne02, ne03, ne12, ne13, nthreads)
    return out.reshape(ne13, ne12, N, M) if (ne12 * ne13) > 1 else out.reshape(N, M)


def mul_mat_id(fmt, mode, w_rows, x, ids, seed=7, nthreads=1):
    """MUL_MAT_ID: w_rows codes [n_expert][M][K], x codes [n_tokens][ne11][K],
    ids int32 [n_tokens][n_used]; returns (codes [n_tokens][n_used][M], number
    of out-of-range ids)."""
    n_expert, M, K = w_rows.shape
    n_tokens, ne11 = x.shape[0], x.shape[1]
    ids = np.ascontiguousarray(ids, np.int32)
    n_used = ids.shape[1]
    dt = np.uint16 if fmt == 16 else np.uint32
    w = np.ascontiguousarray(w_rows, dt).reshape(-1)
    xx = np.ascontiguousarray(x, dt).reshape(-1)
    out = np.empty(n_tokens * n_used * M, dt)
    if fmt == 16:
        bad = lib().orc16_mul_mat_id(MODE[mode], w, xx, ids.reshape(-1), out, K, M, n_expert, ne11, n_used, n_tokens,
                                     n_used, seed, nthreads)
    else:
        bad = lib().orc32_mul_mat_id(w, xx, ids.reshape(-1), out, K, M, n_expert, ne11, n_used, n_tokens, n_used,
                                     nthreads)
    return out.reshape(n_tokens, n_used, M), bad


def soft_max16(mode, src, shape, mask=None, mask_shape=None, scale_code=0x4000, seed=7, nthreads=1):
    s = np.ascontiguousarray(src, np.uint16).reshape(-1)
    out = np.empty_like(s)
    m = None if mask is None else np.ascontiguousarray(mask, np.uint16).reshape(-1)
    lib().orc16_soft_max(MODE[mode], s, _ne(shape), None if m is None else m.ctypes.data_as(ctypes.c_void_p),
                         _ne(mask_shape or (1, 1, 1, 1)), scale_code, out, seed, nthreads)
    return out


def soft_max32(src, shape, mask=None, mask_shape=None, scale_code=0x40000000, nthreads=1):
    s = np.ascontiguousarray(src, np.uint32).reshape(-1)
    out = np.empty_like(s)
    m = None if mask is None else np.ascontiguousarray(mask, np.uint32).reshape(-1)
    lib().orc32_soft_max(s, _ne(shape), None if m is None else m.ctypes.data_as(ctypes.c_void_p),
                         _ne(mask_shape or (1, 1, 1, 1)), scale_code, out, nthreads)
    return out


def rms_norm16(mode, src, ncols, nrows, eps, seed=7, nthreads=1):
    s = np.ascontiguousarray(src, np.uint16).reshape(-1)
    out = np.empty_like(s)
    lib().orc16_rms_norm(MODE[mode], s, out, ncols, nrows, eps, seed, nthreads)
    return out


def rms_norm32(src, ncols, nrows, eps, nthreads=1):
    s = np.ascontiguousarray(src, np.uint32).reshape(-1)
    out = np.empty_like(s)
    lib().orc32_rms_norm(s, out, ncols, nrows, eps, nthreads)
    return out


def mask16(m):
    m = np.ascontiguousarray(m, np.float32)
    return np.array([lib().orc16_mask_from_f32(float(v)) for v in m.ravel()], np.uint16).reshape(m.shape)


def mask32(m):
    m = np.ascontiguousarray(m, np.float32)
    return np.array([lib().orc32_mask_from_f32(float(v)) for v in m.ravel()], np.uint32).reshape(m.shape)


def lfsr_jump(s, n):
    return lib().orc_lfsr_jump(s, n)


def synthstat(config, dist, K, seed=1):
    """the reference's synthetic dot-product error statistics (dot-bench.cpp
    synth(), run.py defaults) replayed through this oracle's mul_mat
    (oracle/synthstat.cpp): {"acc", "acc_l2scale", "total"} each with bias,
    sd, rms, mean_abs, rel_l2"""
    import json
    exe = os.path.join(os.path.dirname(PINCHECK), "synthstat")
    if not os.path.exists(exe):
        build()
    out = subprocess.run([exe, config, dist, str(K), str(seed)], capture_output=True, text=True, check=True).stdout
    return json.loads(out)


def convstat(fmt, n=4194304, order=1):
    """the reference's conversion statistics (dot-bench.cpp convert()) replayed
    through this oracle's conversions (oracle/convstat.cpp); order 1 draws the
    sign before the exponent"""
    import json
    exe = os.path.join(os.path.dirname(PINCHECK), "convstat")
    if not os.path.exists(exe):
        build()
    return json.loads(subprocess.run([exe, str(fmt), str(n), str(order)], capture_output=True, text=True,
                                     check=True).stdout)


def pincheck():
    import json
    if not os.path.exists(PINCHECK):
        build()
    out = json.loads(subprocess.run([PINCHECK], capture_output=True, text=True, check=True).stdout)
    standalone = {k: out.pop(k) for k in ("two_term", "ones", "long_dot", "rms_standalone")}
    out["standalone"] = standalone
    return out


# ---- ggml storage types of weights (test restatement of ggml's block
# layouts and its reference dequantisers; float steps as plain float32
# multiplies and subtractions, in that order) ----
GGML_TYPES = {"f32": 0, "f16": 1, "q4_0": 2, "q8_0": 8, "q4_k": 12, "q6_k": 14, "bf16": 30}
BLOCK = {"f32": (1, 4), "f16": (1, 2), "bf16": (1, 2), "q8_0": (32, 34), "q4_0": (32, 18), "q4_k": (256, 144),
         "q6_k": (256, 210)}


def _f16(b, off):
    return b[:, off:off + 2].copy().view(np.float16).astype(np.float32)[:, 0]


def dequant(type, raw, rows, cols):
    """raw: uint8 [rows][row_bytes] -> float32 [rows][cols]"""
    qk, bb = BLOCK[type]
    nb = cols // qk
    raw = np.ascontiguousarray(raw, np.uint8).reshape(rows, -1)
    if type == "f32":
        return raw.view(np.float32).reshape(rows, cols).copy()
    if type == "f16":
        return raw.view(np.float16).astype(np.float32).reshape(rows, cols)
    if type == "bf16":
        return (raw.view(np.uint16).astype(np.uint32) << 16).view(np.float32).reshape(rows, cols)
    out = np.empty((rows, cols), np.float32)
    for i in range(nb):
        b = raw[:, i * bb:(i + 1) * bb]
        y = out[:, i * qk:(i + 1) * qk]
        if type == "q8_0":
            y[:] = b[:, 2:34].view(np.int8).astype(np.float32) * _f16(b, 0)[:, None]
        elif type == "q4_0":
            d = _f16(b, 0)[:, None]
            qs = b[:, 2:18].astype(np.int32)
            y[:, :16] = ((qs & 0xF) - 8).astype(np.float32) * d
            y[:, 16:] = ((qs >> 4) - 8).astype(np.float32) * d
        elif type == "q4_k":
            d, dmin = _f16(b, 0), _f16(b, 2)
            sc = b[:, 4:16].astype(np.int32)
            qs = b[:, 16:144].astype(np.int32)
            for j in range(8):
                if j < 4:
                    s, m = sc[:, j] & 63, sc[:, j + 4] & 63
                else:
                    s = (sc[:, j + 4] & 0xF) | ((sc[:, j - 4] >> 6) << 4)
                    m = (sc[:, j + 4] >> 4) | ((sc[:, j] >> 6) << 4)
                d1 = (d * s.astype(np.float32))[:, None]
                m1 = (dmin * m.astype(np.float32))[:, None]
                q = qs[:, (j // 2) * 32:(j // 2) * 32 + 32]
                q = (q & 0xF) if j % 2 == 0 else (q >> 4)
                y[:, j * 32:(j + 1) * 32] = d1 * q.astype(np.float32) - m1
        elif type == "q6_k":
            d = _f16(b, 208)
            for n in range(2):
                ql = b[:, n * 64:(n + 1) * 64].astype(np.int32)
                qh = b[:, 128 + n * 32:128 + (n + 1) * 32].astype(np.int32)
                sc = b[:, 192 + n * 8:192 + (n + 1) * 8].view(np.int8).astype(np.float32)
                l = np.arange(32)
                qs = [((ql[:, l] & 0xF) | (((qh[:, l] >> 0) & 3) << 4)) - 32,
                      ((ql[:, l + 32] & 0xF) | (((qh[:, l] >> 2) & 3) << 4)) - 32,
                      ((ql[:, l] >> 4) | (((qh[:, l] >> 4) & 3) << 4)) - 32,
                      ((ql[:, l + 32] >> 4) | (((qh[:, l] >> 6) & 3) << 4)) - 32]
                for quarter in range(4):
                    s = sc[:, (l // 16) + 2 * quarter]
                    y[:, n * 128 + quarter * 32:n * 128 + quarter * 32 + 32] = (d[:, None] * s) * qs[quarter].astype(np.float32)
    return out
