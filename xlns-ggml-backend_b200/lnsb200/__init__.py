"""Host-side mirror of the reference's lns_cuda::kernel_set
(lns-backend/cuda/lns-cuda-kernels.h:85-139) over the C ABI of
include/lnsb200.h.

One KernelSet per (summation-mode build, format), like the reference's
xlns16_kernels() / xlns32_kernels().  Tensors are torch CUDA tensors used
purely as device memory: uint16 (xlns16 codes), int32 (xlns32 codes, same
bits as uint32) or float32.  Every call launches asynchronously on the
current torch stream (or the given one) and raises LnsbError on failure --
there is no CPU fallback.
"""
import ctypes

from . import _lib
from ._lib import MODES, XLNS16, XLNS32, LnsbError, MulMatArgs, Shape4, SoftMaxArgs  # noqa: F401

__all__ = ["KernelSet", "MODES", "XLNS16", "XLNS32", "LnsbError", "MulMatArgs", "SoftMaxArgs", "Shape4",
           "kernels", "monte_get_state", "monte_set_state", "monte_reserve"]


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(stream):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _shape4(shape):
    ne = list(shape) + [1] * (4 - len(shape))
    return Shape4((ctypes.c_int64 * 4)(*ne))


class KernelSet:
    """kernel_set for one format of one summation-mode build."""

    def __init__(self, fmt=XLNS16, mode="base"):
        if fmt not in (XLNS16, XLNS32):
            raise ValueError("format must be 16 or 32")
        self.fmt = fmt
        self.mode = mode
        self.lib = _lib.load(mode)

    # ---- identity (kernel_set::format_name ... monte_impl) ----
    def format_name(self):
        return self.lib.lnsb_format_name(self.fmt).decode()

    def value_size(self):
        return self.lib.lnsb_value_size(self.fmt)

    def sum_mode(self):
        r = self.lib.lnsb_sum_mode(self.fmt)
        return r.decode() if r else None

    def monte_impl(self):
        r = self.lib.lnsb_monte_impl(self.fmt)
        return r.decode() if r else None

    def description(self):
        return self.lib.lnsb_description(self.fmt).decode()

    # ---- draw accounting ----
    def mul_mat_draws(self, K, M, N, ne02=1, ne03=1, ne12=1, ne13=1):
        a = MulMatArgs(None, None, None, K, M, N, ne02, ne03, ne12, ne13, 0)
        return self.lib.lnsb_mul_mat_draws(self.fmt, ctypes.byref(a))

    def soft_max_draws(self, ncols, nrows):
        return self.lib.lnsb_soft_max_draws(self.fmt, ncols, nrows)

    def rms_norm_draws(self, ncols, nrows):
        return self.lib.lnsb_rms_norm_draws(self.fmt, ncols, nrows)

    # ---- tables / conversions ----
    def upload_tables(self):
        _lib.check(self.lib, "lnsb_upload_tables", self.lib.lnsb_upload_tables(self.fmt))

    def add_latency(self, kind, lanes=32, steps=4096):
        """SM cycles of one dependent LNS addition (lnsb_add_latency): kind 0 the
        key-form xlns16 addition of the latency mul_mat kernels, 1 / 2 the
        non-negative xlns16 / xlns32 additions of the normalisers, 3 the
        general xlns32 addition of the latency mat-vecs (sum32, xlns32)"""
        import torch
        out = torch.zeros(2, dtype=torch.int64, device="cuda")
        _lib.check(self.lib, "lnsb_add_latency", self.lib.lnsb_add_latency(kind, lanes, steps, _ptr(out), None))
        torch.cuda.synchronize()
        return out[0].item() / (steps - 1)

    def to_lns(self, src, dst, stream=None):
        _lib.check(self.lib, "lnsb_to_lns", self.lib.lnsb_to_lns(self.fmt, _ptr(src), _ptr(dst), src.numel(), _stream(stream)))

    def to_lns_transposed(self, src, dst, rows, cols, dst_ld, stream=None):
        _lib.check(self.lib, "lnsb_to_lns_transposed",
                   self.lib.lnsb_to_lns_transposed(self.fmt, _ptr(src), _ptr(dst), rows, cols, dst_ld, _stream(stream)))

    def to_f32(self, src, dst, stream=None):
        _lib.check(self.lib, "lnsb_to_f32", self.lib.lnsb_to_f32(self.fmt, _ptr(src), _ptr(dst), src.numel(), _stream(stream)))

    # ---- the hot path ----
    def _mm_args(self, w, x, dst, K, M, N, slices, monte_seed):
        ne02, ne03, ne12, ne13 = slices
        return MulMatArgs(w.data_ptr(), x.data_ptr(), dst.data_ptr() if dst is not None else None,
                          K, M, N, ne02, ne03, ne12, ne13, monte_seed)

    def mul_mat(self, w, x, dst, K, M, N, slices=(1, 1, 1, 1), monte_seed=7, stream=None):
        """dst (F32, [slices][N][M]) = W^T x; w k-major [K][M] per weight slice, x [N][K]."""
        a = self._mm_args(w, x, dst, K, M, N, slices, monte_seed)
        _lib.check(self.lib, "lnsb_mul_mat", self.lib.lnsb_mul_mat(self.fmt, ctypes.byref(a), _stream(stream)))

    def mul_mat_xf32(self, w, x_f32, x_work, dst, K, M, N, slices=(1, 1, 1, 1), monte_seed=7, stream=None):
        """the MUL_MAT op over F32 activations (lnsb_mul_mat_xf32): x_f32 [N][K] floats, converted as
        the kernel stages them or into x_work (N*K codes) first; dst F32 as mul_mat"""
        a = self._mm_args(w, x_f32, dst, K, M, N, slices, monte_seed)
        _lib.check(self.lib, "lnsb_mul_mat_xf32",
                   self.lib.lnsb_mul_mat_xf32(self.fmt, ctypes.byref(a), _ptr(x_work), _stream(stream)))

    def mul_mat_lns(self, w, x, dst, K, M, N, slices=(1, 1, 1, 1), monte_seed=7, stream=None):
        """as mul_mat with LNS codes out"""
        a = self._mm_args(w, x, None, K, M, N, slices, monte_seed)
        _lib.check(self.lib, "lnsb_mul_mat_lns", self.lib.lnsb_mul_mat_lns(self.fmt, ctypes.byref(a), _ptr(dst), _stream(stream)))

    def attn_decode(self, q, k_cache, v_cache, kv_ld, nkv, n_head, n_head_kv, head_dim, scale, dst, monte_seed=7,
                    stream=None, dst_lns=None):
        """one decode step's attention (lnsb_attn_decode): q F32 [n_head][head_dim], caches F16
        [nkv][kv_ld], dst F32 [n_head][head_dim] (or None), dst_lns its codes (optional)"""
        a = _lib.AttnDecodeArgs(_ptr(q), _ptr(k_cache), _ptr(v_cache), kv_ld, nkv, n_head, n_head_kv, head_dim, scale,
                                _ptr(dst) if dst is not None else None, monte_seed,
                                _ptr(dst_lns) if dst_lns is not None else None)
        _lib.check(self.lib, "lnsb_attn_decode", self.lib.lnsb_attn_decode(self.fmt, ctypes.byref(a), _stream(stream)))

    def norm_block(self, src, dst_lns, ncols, nrows, eps, residual=None, x_out=None, weight=None, monte_seed=7,
                   stream=None):
        """lnsb_norm_block: [residual add,] rms_norm, [times weight,] to_lns"""
        opt = lambda t: _ptr(t) if t is not None else None
        a = _lib.NormBlockArgs(_ptr(src), opt(residual), opt(x_out), opt(weight), _ptr(dst_lns), ncols, nrows, eps,
                               monte_seed)
        _lib.check(self.lib, "lnsb_norm_block", self.lib.lnsb_norm_block(self.fmt, ctypes.byref(a), _stream(stream)))

    def glu_lns(self, gate, up, gate_stride, up_stride, dst_lns, ncols, nrows, op="swiglu", stream=None):
        _lib.check(self.lib, "lnsb_glu_lns", self.lib.lnsb_glu_lns(self.fmt, 0 if op == "swiglu" else 1, _ptr(gate),
                                                                   _ptr(up), gate_stride, up_stride, _ptr(dst_lns),
                                                                   ncols, nrows, _stream(stream)))

    def rope_qkv(self, qkv, ld, cos_sin, n_dims, n_head, n_head_kv, head_dim, n_tokens, q_out, k_cache, v_cache, kv_ld,
                 neox=False, stream=None):
        a = _lib.RopeQkvArgs(_ptr(qkv), ld, _ptr(cos_sin), n_dims, 1 if neox else 0, n_head, n_head_kv, head_dim,
                             n_tokens, _ptr(q_out), _ptr(k_cache), _ptr(v_cache), kv_ld)
        _lib.check(self.lib, "lnsb_rope_qkv", self.lib.lnsb_rope_qkv(self.fmt, ctypes.byref(a), _stream(stream)))

    def attn_decode_max_keys(self, head_dim):
        return self.lib.lnsb_attn_decode_max_keys(self.fmt, head_dim)

    def type_row_bytes(self, type, cols):
        return self.lib.lnsb_type_row_bytes(_lib.TYPES.get(type, type), cols)

    def to_lns_transposed_typed(self, type, src, dst, rows, cols, dst_ld, stream=None):
        """dst[c * dst_ld + r] = lns(value c of row r); src rows in a ggml storage type (name or id)"""
        _lib.check(self.lib, "lnsb_to_lns_transposed_typed",
                   self.lib.lnsb_to_lns_transposed_typed(self.fmt, _lib.TYPES.get(type, type), _ptr(src), _ptr(dst),
                                                         rows, cols, dst_ld, _stream(stream)))

    def dequantize(self, type, src, dst, rows, cols, stream=None):
        _lib.check(self.lib, "lnsb_dequantize",
                   self.lib.lnsb_dequantize(_lib.TYPES.get(type, type), _ptr(src), _ptr(dst), rows, cols, _stream(stream)))

    def mul_mat_lns_peers(self, w, x, ptrs_dev, n_peers, ld, offset, K, M, N, slices=(1, 1, 1, 1), monte_seed=7,
                          stream=None):
        """mul_mat with the output-row all-gather fused into the store: codes
        into every peer buffer (ptrs_dev: device address of an array of
        n_peers pointers) at [N][ld] columns [offset, offset + M)"""
        a = self._mm_args(w, x, None, K, M, N, slices, monte_seed)
        p = _lib.PeerOut(ptrs_dev, n_peers, ld, offset)
        _lib.check(self.lib, "lnsb_mul_mat_lns_peers",
                   self.lib.lnsb_mul_mat_lns_peers(self.fmt, ctypes.byref(a), ctypes.byref(p), _stream(stream)))

    def _mmid_args(self, w, x, ids, dst, K, M, n_expert, ne11, n_used, n_tokens, monte_seed):
        return _lib.MulMatIdArgs(w.data_ptr(), x.data_ptr(), ids.data_ptr(), dst.data_ptr() if dst is not None else None,
                                 K, M, n_expert, ne11, n_used, n_tokens, n_used, monte_seed)

    def mul_mat_id(self, w, x, ids, dst, K, M, n_expert, ne11, n_used, n_tokens, monte_seed=7, stream=None):
        """MUL_MAT_ID: dst (F32, [n_tokens][n_used][M]); w k-major [n_expert][K][M],
        x [n_tokens][ne11][K], ids int32 [n_tokens][n_used] on the device."""
        a = self._mmid_args(w, x, ids, dst, K, M, n_expert, ne11, n_used, n_tokens, monte_seed)
        _lib.check(self.lib, "lnsb_mul_mat_id", self.lib.lnsb_mul_mat_id(self.fmt, ctypes.byref(a), _stream(stream)))

    def mul_mat_id_lns(self, w, x, ids, dst, K, M, n_expert, ne11, n_used, n_tokens, monte_seed=7, stream=None):
        a = self._mmid_args(w, x, ids, None, K, M, n_expert, ne11, n_used, n_tokens, monte_seed)
        _lib.check(self.lib, "lnsb_mul_mat_id_lns",
                   self.lib.lnsb_mul_mat_id_lns(self.fmt, ctypes.byref(a), _ptr(dst), _stream(stream)))

    def mul_mat_id_draws(self, K, M, n_used, n_tokens):
        a = _lib.MulMatIdArgs(None, None, None, None, K, M, 1, 1, n_used, n_tokens, n_used, 0)
        return self.lib.lnsb_mul_mat_id_draws(self.fmt, ctypes.byref(a))

    def mul_mat_id_bad_ids(self):
        """out-of-range ids met on the current device since the last call"""
        c = ctypes.c_int64()
        _lib.check(self.lib, "lnsb_mul_mat_id_bad_ids", self.lib.lnsb_mul_mat_id_bad_ids(ctypes.byref(c)))
        return c.value

    def soft_max(self, src, shape, dst, work, mask=None, mask_shape=None, scale=1.0, monte_seed=7, stream=None):
        a = SoftMaxArgs(src.data_ptr(), _shape4(shape), mask.data_ptr() if mask is not None else None,
                        _shape4(mask_shape or (1, 1, 1, 1)), scale, dst.data_ptr(), work.data_ptr(), monte_seed)
        _lib.check(self.lib, "lnsb_soft_max", self.lib.lnsb_soft_max(self.fmt, ctypes.byref(a), _stream(stream)))

    def soft_max_lns(self, src, shape, dst, work, mask=None, mask_shape=None, scale_code=0x4000, monte_seed=7, stream=None):
        ne = (ctypes.c_int64 * 4)(*(list(shape) + [1] * (4 - len(shape))))
        mne = (ctypes.c_int64 * 4)(*(list(mask_shape) + [1] * (4 - len(mask_shape)))) if mask is not None else None
        _lib.check(self.lib, "lnsb_soft_max_lns",
                   self.lib.lnsb_soft_max_lns(self.fmt, _ptr(src), ne, _ptr(mask), mne, scale_code, _ptr(dst),
                                              _ptr(work), monte_seed, _stream(stream)))

    def rms_norm(self, src, dst, ncols, nrows, eps, monte_seed=7, stream=None):
        _lib.check(self.lib, "lnsb_rms_norm",
                   self.lib.lnsb_rms_norm(self.fmt, _ptr(src), _ptr(dst), ncols, nrows, eps, monte_seed, _stream(stream)))

    def rms_norm_lns(self, src, dst, ncols, nrows, eps, monte_seed=7, stream=None):
        _lib.check(self.lib, "lnsb_rms_norm_lns",
                   self.lib.lnsb_rms_norm_lns(self.fmt, _ptr(src), _ptr(dst), ncols, nrows, eps, monte_seed, _stream(stream)))


    # ---- elementwise ops of the model graph (F32 in and out) ----
    BINARY = {"add": 0, "mul": 1, "div": 2}
    UNARY = {"silu": 0, "gelu": 1, "relu": 2, "tanh": 3}

    def binary(self, op, a, a_shape, b, b_shape, dst, stream=None):
        """dst = a op b, b repeated to a's shape; shapes ggml order (ne0 innermost)"""
        ane, bne = _shape4(a_shape).ne, _shape4(b_shape).ne
        _lib.check(self.lib, "lnsb_binary", self.lib.lnsb_binary(self.fmt, self.BINARY[op], _ptr(a), ane, _ptr(b), bne,
                                                                 _ptr(dst), _stream(stream)))

    def scale(self, src, dst, n, s, b=0.0, stream=None):
        _lib.check(self.lib, "lnsb_scale", self.lib.lnsb_scale(self.fmt, _ptr(src), _ptr(dst), n, s, b, _stream(stream)))

    def unary(self, op, src, dst, n, stream=None):
        _lib.check(self.lib, "lnsb_unary", self.lib.lnsb_unary(self.fmt, self.UNARY[op], _ptr(src), _ptr(dst), n,
                                                               _stream(stream)))

    def glu(self, gate, up, gate_stride, up_stride, dst, ncols, nrows, op="swiglu", stream=None):
        _lib.check(self.lib, "lnsb_glu", self.lib.lnsb_glu(self.fmt, 0 if op == "swiglu" else 1, _ptr(gate), _ptr(up),
                                                           gate_stride, up_stride, _ptr(dst), ncols, nrows, _stream(stream)))

    def rope(self, src, shape, cos_sin, n_dims, dst, neox=False, stream=None):
        a = _lib.RopeArgs(_ptr(src), _shape4(shape), _ptr(cos_sin), n_dims, 1 if neox else 0, _ptr(dst))
        _lib.check(self.lib, "lnsb_rope", self.lib.lnsb_rope(self.fmt, ctypes.byref(a), _stream(stream)))

    def f32_to_f16(self, src, dst, n, stream=None):
        _lib.check(self.lib, "lnsb_f32_to_f16", self.lib.lnsb_f32_to_f16(_ptr(src), _ptr(dst), n, _stream(stream)))

    def f16_to_f32(self, src, dst, n, stream=None):
        _lib.check(self.lib, "lnsb_f16_to_f32", self.lib.lnsb_f16_to_f32(_ptr(src), _ptr(dst), n, _stream(stream)))


def kernels(fmt=XLNS16, mode="base"):
    return KernelSet(fmt, mode)


# ---- Monte state (ggml-lns.h:13-24): process-wide, per monte build ----
def monte_get_state(mode="monte"):
    lib = _lib.load(mode)
    s = ctypes.c_uint16()
    _lib.check(lib, "lnsb_monte_get_state", lib.lnsb_monte_get_state(ctypes.byref(s)))
    return s.value


def monte_set_state(state, mode="monte"):
    lib = _lib.load(mode)
    _lib.check(lib, "lnsb_monte_set_state", lib.lnsb_monte_set_state(state))


def monte_reserve(draws, mode="monte"):
    lib = _lib.load(mode)
    s = ctypes.c_uint16()
    _lib.check(lib, "lnsb_monte_reserve", lib.lnsb_monte_reserve(draws, ctypes.byref(s)))
    return s.value


class WeightCache:
    """lnsb_weight_cache_*: weights converted to LNS once per (data pointer,
    type, rows, cols) and kept on the device within a byte budget
    (budget < 0: GGML_LNS_CUDA_CACHE_MB, else free memory less 1 GiB)."""

    def __init__(self, ks, budget=-1):
        self.ks = ks
        self.lib = ks.lib
        self.h = self.lib.lnsb_weight_cache_create(ks.fmt, budget)
        if not self.h:
            raise LnsbError(self.lib, "lnsb_weight_cache_create", -1)

    def get(self, src, type, rows, cols, scratch=None, stream=None):
        """device address of the k-major LNS image of `src` (a torch tensor
        on the device, or a numpy array / address in host memory)"""
        out = ctypes.c_void_p()
        _lib.check(self.lib, "lnsb_weight_cache_get",
                   self.lib.lnsb_weight_cache_get(self.h, _addr(src), _lib.TYPES.get(type, type), rows, cols,
                                                  _ptr(scratch) if scratch is not None else None, ctypes.byref(out),
                                                  _stream(stream)))
        return out.value

    def stats(self):
        e, u, b = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
        _lib.check(self.lib, "lnsb_weight_cache_stats",
                   self.lib.lnsb_weight_cache_stats(self.h, ctypes.byref(e), ctypes.byref(u), ctypes.byref(b)))
        return {"entries": e.value, "used": u.value, "budget": b.value}

    def close(self):
        if self.h:
            self.lib.lnsb_weight_cache_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _addr(obj):
    """device or host address of a torch tensor, a numpy array or an int"""
    if hasattr(obj, "data_ptr"):
        return obj.data_ptr()
    if hasattr(obj, "ctypes"):
        return obj.ctypes.data
    return int(obj)
