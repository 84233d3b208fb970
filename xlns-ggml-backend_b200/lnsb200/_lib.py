"""ctypes binding of include/lnsb200.h -- the exact calls a maintainer's FFI
would make.  Loading fails loudly when the built library is missing: there is
no CPU fallback anywhere in this package."""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_DIR = os.path.join(os.path.dirname(HERE), "lib")

MODES = ("base", "monte", "monte_bylpvip", "lpvip", "sum32")

# ggml storage types of weights (ggml_type ids)
TYPES = {"f32": 0, "f16": 1, "q4_0": 2, "q8_0": 8, "q4_k": 12, "q6_k": 14, "bf16": 30}

XLNS16 = 16
XLNS32 = 32

STATUS = {0: "LNSB_OK", -1: "LNSB_E_INVALID", -2: "LNSB_E_NO_TABLES", -3: "LNSB_E_UNSUPPORTED",
          -4: "LNSB_E_TOO_LARGE", -5: "LNSB_E_NO_DEVICE"}


class Shape4(ctypes.Structure):
    _fields_ = [("ne", ctypes.c_int64 * 4)]


class MulMatArgs(ctypes.Structure):
    _fields_ = [("w", ctypes.c_void_p), ("x", ctypes.c_void_p), ("dst", ctypes.c_void_p),
                ("K", ctypes.c_int64), ("M", ctypes.c_int64), ("N", ctypes.c_int64),
                ("ne02", ctypes.c_int64), ("ne03", ctypes.c_int64), ("ne12", ctypes.c_int64), ("ne13", ctypes.c_int64),
                ("monte_seed", ctypes.c_uint16)]


class MulMatIdArgs(ctypes.Structure):
    _fields_ = [("w", ctypes.c_void_p), ("x", ctypes.c_void_p), ("ids", ctypes.c_void_p), ("dst", ctypes.c_void_p),
                ("K", ctypes.c_int64), ("M", ctypes.c_int64), ("n_expert", ctypes.c_int64), ("ne11", ctypes.c_int64),
                ("n_used", ctypes.c_int64), ("n_tokens", ctypes.c_int64), ("ids_stride", ctypes.c_int64),
                ("monte_seed", ctypes.c_uint16)]


class AttnDecodeArgs(ctypes.Structure):
    _fields_ = [("q", ctypes.c_void_p), ("k_cache", ctypes.c_void_p), ("v_cache", ctypes.c_void_p),
                ("kv_ld", ctypes.c_int64), ("nkv", ctypes.c_int64), ("n_head", ctypes.c_int), ("n_head_kv", ctypes.c_int),
                ("head_dim", ctypes.c_int), ("scale", ctypes.c_float), ("dst", ctypes.c_void_p),
                ("monte_seed", ctypes.c_uint16), ("dst_lns", ctypes.c_void_p)]


class NormBlockArgs(ctypes.Structure):
    _fields_ = [("src", ctypes.c_void_p), ("residual", ctypes.c_void_p), ("x_out", ctypes.c_void_p),
                ("weight", ctypes.c_void_p), ("dst_lns", ctypes.c_void_p), ("ncols", ctypes.c_int64),
                ("nrows", ctypes.c_int64), ("eps", ctypes.c_float), ("monte_seed", ctypes.c_uint16)]


class RopeQkvArgs(ctypes.Structure):
    _fields_ = [("qkv", ctypes.c_void_p), ("ld", ctypes.c_int64), ("cos_sin", ctypes.c_void_p), ("n_dims", ctypes.c_int),
                ("neox", ctypes.c_int), ("n_head", ctypes.c_int), ("n_head_kv", ctypes.c_int), ("head_dim", ctypes.c_int),
                ("n_tokens", ctypes.c_int64), ("q_out", ctypes.c_void_p), ("k_cache", ctypes.c_void_p),
                ("v_cache", ctypes.c_void_p), ("kv_ld", ctypes.c_int64)]


class PeerOut(ctypes.Structure):
    _fields_ = [("ptrs", ctypes.c_void_p), ("n", ctypes.c_int), ("ld", ctypes.c_int64), ("offset", ctypes.c_int64)]


class SoftMaxArgs(ctypes.Structure):
    _fields_ = [("src", ctypes.c_void_p), ("src_shape", Shape4), ("mask", ctypes.c_void_p), ("mask_shape", Shape4),
                ("scale", ctypes.c_float), ("dst", ctypes.c_void_p), ("work", ctypes.c_void_p),
                ("monte_seed", ctypes.c_uint16)]


class RopeArgs(ctypes.Structure):
    _fields_ = [("src", ctypes.c_void_p), ("shape", Shape4), ("cos_sin", ctypes.c_void_p), ("n_dims", ctypes.c_int),
                ("neox", ctypes.c_int), ("dst", ctypes.c_void_p)]


# (name, restype, argtypes) for every function of include/lnsb200.h
_I64 = ctypes.c_int64
_VP = ctypes.c_void_p
SIGNATURES = [
    ("lnsb_format_name", ctypes.c_char_p, [ctypes.c_int]),
    ("lnsb_value_size", ctypes.c_size_t, [ctypes.c_int]),
    ("lnsb_sum_mode", ctypes.c_char_p, [ctypes.c_int]),
    ("lnsb_monte_impl", ctypes.c_char_p, [ctypes.c_int]),
    ("lnsb_description", ctypes.c_char_p, [ctypes.c_int]),
    ("lnsb_mul_mat_draws", ctypes.c_uint64, [ctypes.c_int, ctypes.POINTER(MulMatArgs)]),
    ("lnsb_soft_max_draws", ctypes.c_uint64, [ctypes.c_int, _I64, _I64]),
    ("lnsb_rms_norm_draws", ctypes.c_uint64, [ctypes.c_int, _I64, _I64]),
    ("lnsb_upload_tables", ctypes.c_int, [ctypes.c_int]),
    ("lnsb_to_lns", ctypes.c_int, [ctypes.c_int, _VP, _VP, _I64, _VP]),
    ("lnsb_to_lns_transposed", ctypes.c_int, [ctypes.c_int, _VP, _VP, _I64, _I64, _I64, _VP]),
    ("lnsb_to_f32", ctypes.c_int, [ctypes.c_int, _VP, _VP, _I64, _VP]),
    ("lnsb_type_row_bytes", ctypes.c_size_t, [ctypes.c_int, _I64]),
    ("lnsb_to_lns_transposed_typed", ctypes.c_int, [ctypes.c_int, ctypes.c_int, _VP, _VP, _I64, _I64, _I64, _VP]),
    ("lnsb_dequantize", ctypes.c_int, [ctypes.c_int, _VP, _VP, _I64, _I64, _VP]),
    ("lnsb_weight_cache_create", _VP, [ctypes.c_int, _I64]),
    ("lnsb_weight_cache_destroy", None, [_VP]),
    ("lnsb_weight_cache_get", ctypes.c_int, [_VP, _VP, ctypes.c_int, _I64, _I64, _VP, ctypes.POINTER(_VP), _VP]),
    ("lnsb_weight_cache_stats", ctypes.c_int, [_VP, ctypes.POINTER(_I64), ctypes.POINTER(_I64), ctypes.POINTER(_I64)]),
    ("lnsb_mul_mat", ctypes.c_int, [ctypes.c_int, ctypes.POINTER(MulMatArgs), _VP]),
    ("lnsb_mul_mat_lns", ctypes.c_int, [ctypes.c_int, ctypes.POINTER(MulMatArgs), _VP, _VP]),
    ("lnsb_mul_mat_xf32", ctypes.c_int, [ctypes.c_int, ctypes.POINTER(MulMatArgs), _VP, _VP]),
    ("lnsb_mul_mat_lns_peers", ctypes.c_int, [ctypes.c_int, ctypes.POINTER(MulMatArgs), ctypes.POINTER(PeerOut), _VP]),
    ("lnsb_group_barrier", ctypes.c_int, [_VP, ctypes.c_int, ctypes.c_int, ctypes.c_int32, _VP, _VP]),
    ("lnsb_add_latency", ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_int, _VP, _VP]),
    ("lnsb_mul_mat_id", ctypes.c_int, [ctypes.c_int, ctypes.POINTER(MulMatIdArgs), _VP]),
    ("lnsb_mul_mat_id_lns", ctypes.c_int, [ctypes.c_int, ctypes.POINTER(MulMatIdArgs), _VP, _VP]),
    ("lnsb_mul_mat_id_draws", ctypes.c_uint64, [ctypes.c_int, ctypes.POINTER(MulMatIdArgs)]),
    ("lnsb_mul_mat_id_bad_ids", ctypes.c_int, [ctypes.POINTER(_I64)]),
    ("lnsb_soft_max", ctypes.c_int, [ctypes.c_int, ctypes.POINTER(SoftMaxArgs), _VP]),
    ("lnsb_soft_max_lns", ctypes.c_int, [ctypes.c_int, _VP, ctypes.POINTER(_I64), _VP, ctypes.POINTER(_I64),
                                         ctypes.c_uint32, _VP, _VP, ctypes.c_uint16, _VP]),
    ("lnsb_soft_max_lns_noalloc", ctypes.c_int, [ctypes.c_int, _VP, ctypes.POINTER(_I64), _VP, ctypes.POINTER(_I64),
                                                 ctypes.c_uint32, _VP, ctypes.c_uint16, _VP]),
    ("lnsb_rms_norm", ctypes.c_int, [ctypes.c_int, _VP, _VP, _I64, _I64, ctypes.c_float, ctypes.c_uint16, _VP]),
    ("lnsb_rms_norm_lns", ctypes.c_int, [ctypes.c_int, _VP, _VP, _I64, _I64, ctypes.c_float, ctypes.c_uint16, _VP]),
    ("lnsb_binary", ctypes.c_int, [ctypes.c_int, ctypes.c_int, _VP, ctypes.POINTER(_I64), _VP, ctypes.POINTER(_I64),
                                   _VP, _VP]),
    ("lnsb_scale", ctypes.c_int, [ctypes.c_int, _VP, _VP, _I64, ctypes.c_float, ctypes.c_float, _VP]),
    ("lnsb_unary", ctypes.c_int, [ctypes.c_int, ctypes.c_int, _VP, _VP, _I64, _VP]),
    ("lnsb_glu", ctypes.c_int, [ctypes.c_int, ctypes.c_int, _VP, _VP, _I64, _I64, _VP, _I64, _I64, _VP]),
    ("lnsb_rope", ctypes.c_int, [ctypes.c_int, ctypes.POINTER(RopeArgs), _VP]),
    ("lnsb_attn_decode", ctypes.c_int, [ctypes.c_int, ctypes.POINTER(AttnDecodeArgs), _VP]),
    ("lnsb_attn_decode_max_keys", _I64, [ctypes.c_int, ctypes.c_int]),
    ("lnsb_norm_block", ctypes.c_int, [ctypes.c_int, ctypes.POINTER(NormBlockArgs), _VP]),
    ("lnsb_glu_lns", ctypes.c_int, [ctypes.c_int, ctypes.c_int, _VP, _VP, _I64, _I64, _VP, _I64, _I64, _VP]),
    ("lnsb_rope_qkv", ctypes.c_int, [ctypes.c_int, ctypes.POINTER(RopeQkvArgs), _VP]),
    ("lnsb_f32_to_f16", ctypes.c_int, [_VP, _VP, _I64, _VP]),
    ("lnsb_f16_to_f32", ctypes.c_int, [_VP, _VP, _I64, _VP]),
    ("lnsb_monte_get_state", ctypes.c_int, [ctypes.POINTER(ctypes.c_uint16)]),
    ("lnsb_monte_set_state", ctypes.c_int, [ctypes.c_uint16]),
    ("lnsb_monte_reserve", ctypes.c_int, [ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint16)]),
    ("lnsb_error_string", ctypes.c_char_p, [ctypes.c_int]),
]

_loaded = {}


def lib_path(mode):
    return os.path.join(LIB_DIR, "liblnsb200_%s.so" % mode)


def load(mode="base"):
    """The C-ABI library of one summation-mode build (loaded once)."""
    if mode not in MODES:
        raise ValueError("unknown summation mode %r (one of %s)" % (mode, ", ".join(MODES)))
    if mode in _loaded:
        return _loaded[mode]
    path = lib_path(mode)
    if not os.path.exists(path):
        raise RuntimeError("LNS B200 library %s is not built; run `python xlns-ggml-backend_b200/build.py` "
                           "(this package has no CPU fallback)" % path)
    lib = ctypes.CDLL(path, mode=ctypes.RTLD_LOCAL)
    for name, res, args in SIGNATURES:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _loaded[mode] = lib
    return lib


class LnsbError(RuntimeError):
    def __init__(self, lib, fn, status):
        msg = lib.lnsb_error_string(status).decode()
        super().__init__("%s failed: %s (%s)" % (fn, STATUS.get(status, "cudaError %d" % status), msg))
        self.status = status


def check(lib, fn, status):
    if status != 0:
        raise LnsbError(lib, fn, status)
    return status
