"""The ggml backend's host layer (include/lnsb200_graph.h) from Python: the
tensor descriptor, supports_op and its parts, and graph_compute.

A node is a `Tensor` (the C struct lnsb_tensor) describing a torch tensor
(device memory) or a numpy array (host memory): type, shape and byte strides
in ggml's order (ne[0] innermost), the op, its op parameters and its sources.
"""
import ctypes
import struct

from . import _lib

OPS = ["NONE", "RESHAPE", "VIEW", "PERMUTE", "TRANSPOSE", "MUL_MAT", "MUL_MAT_ID", "ADD", "MUL", "DIV", "SCALE",
       "RMS_NORM", "SOFT_MAX", "ROPE", "UNARY", "GLU", "GET_ROWS", "CPY", "CONT"]
OP = {name: i for i, name in enumerate(OPS)}
UNARY = {"silu": 0, "gelu": 1, "relu": 2, "tanh": 3}
GLU = {"swiglu": 0, "geglu": 1}
TYPES = dict(_lib.TYPES, i32=26)
FLAG_COMPUTE, FLAG_WEIGHTS = 1, 2
ROPE_NEOX = 2


class Tensor(ctypes.Structure):
    pass


Tensor._fields_ = [("type", ctypes.c_int32), ("op", ctypes.c_int32), ("ne", ctypes.c_int64 * 4),
                   ("nb", ctypes.c_int64 * 4), ("op_params", ctypes.c_int32 * 16), ("flags", ctypes.c_int32),
                   ("src", ctypes.POINTER(Tensor) * 4), ("data", ctypes.c_void_p), ("name", ctypes.c_char * 64)]

_SIGS = [
    ("lnsb_op_name", ctypes.c_char_p, [ctypes.c_int]),
    ("lnsb_op_desc", ctypes.c_char_p, [ctypes.POINTER(Tensor)]),
    ("lnsb_check_op", ctypes.c_int, [ctypes.c_int, ctypes.POINTER(Tensor), ctypes.POINTER(ctypes.c_char_p)]),
    ("lnsb_resolve_backend_selection", ctypes.c_int, [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_size_t]),
    ("lnsb_backend_selected_by", ctypes.c_int, [ctypes.c_char_p, ctypes.c_char_p]),
    ("lnsb_op_matches", ctypes.c_int, [ctypes.POINTER(Tensor), ctypes.c_char_p]),
    ("lnsb_op_disabled_by", ctypes.c_int, [ctypes.POINTER(Tensor), ctypes.c_char_p, ctypes.c_char_p]),
    ("lnsb_audit_line", ctypes.c_int, [ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(Tensor), ctypes.c_int,
                                       ctypes.c_char_p, ctypes.c_char_p, ctypes.c_size_t]),
    ("lnsb_supports_op", ctypes.c_int, [ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(Tensor)]),
    ("lnsb_device_description", ctypes.c_char_p, [ctypes.c_int]),
    ("lnsb_graph_ctx_create", ctypes.c_void_p, [ctypes.c_int, ctypes.c_int64, ctypes.c_void_p]),
    ("lnsb_graph_ctx_destroy", None, [ctypes.c_void_p]),
    ("lnsb_graph_compute", ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.POINTER(Tensor)), ctypes.c_int,
                                          ctypes.POINTER(ctypes.c_int)]),
    ("lnsb_copy_strided", ctypes.c_int, [ctypes.c_int, ctypes.c_void_p, ctypes.POINTER(ctypes.c_int64),
                                         ctypes.POINTER(ctypes.c_int64), ctypes.c_void_p, ctypes.c_void_p]),
]
_bound = set()


def lib(mode="base"):
    L = _lib.load(mode)
    if id(L) not in _bound:
        for name, res, args in _SIGS:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _bound.add(id(L))
    return L


_TYPE_OF = {"float32": "f32", "float16": "f16", "bfloat16": "bf16", "int32": "i32"}


def _dtype_name(a):
    return str(a.dtype).replace("torch.", "")


def tensor(a=None, type=None, ne=None, nb=None, op="NONE", src=(), params=(), name="", flags=0, data=None):
    """A descriptor.  a: a torch tensor or numpy array (shape in numpy order,
    innermost last; its strides become nb), or None with ne / nb / type given
    (raw rows, e.g. quantised blocks, through `data`)."""
    t = Tensor()
    if a is not None:
        shape = list(a.shape)[::-1]
        esz = a.element_size() if hasattr(a, "element_size") else a.itemsize
        strides = list(a.stride())[::-1] if hasattr(a, "stride") and callable(a.stride) else [s // esz for s in a.strides[::-1]]
        ne = shape + [1] * (4 - len(shape))
        nb = [s * esz for s in strides] + [0] * (4 - len(strides))
        for i in range(len(shape), 4):
            nb[i] = nb[i - 1] * ne[i - 1] if i > 0 else esz
        type = type if type is not None else _TYPE_OF[_dtype_name(a)]
        data = a.data_ptr() if hasattr(a, "data_ptr") else a.ctypes.data
    t.type = TYPES[type] if isinstance(type, str) else type
    t.op = OP[op] if isinstance(op, str) else op
    for i in range(4):
        t.ne[i] = ne[i]
        t.nb[i] = nb[i]
    for i, p in enumerate(params):
        t.op_params[i] = struct.unpack("<i", struct.pack("<f", p))[0] if isinstance(p, float) else p
    t.flags = flags
    for i, s in enumerate(src):
        if s is not None:
            t.src[i] = ctypes.pointer(s)
    t.data = data
    t.name = name.encode()[:63]
    return t


def check(node, fmt=16, mode="base"):
    """(supported, reason) of the predicate alone"""
    r = ctypes.c_char_p()
    ok = lib(mode).lnsb_check_op(fmt, ctypes.byref(node), ctypes.byref(r))
    return bool(ok), (r.value.decode() if r.value else None)


def resolve_selection(value, mode="base"):
    buf = ctypes.create_string_buffer(256)
    lib(mode).lnsb_resolve_backend_selection(value.encode() if value is not None else None, buf, 256)
    return [d for d in buf.value.decode().split(",") if d]


def selected(device, value, mode="base"):
    return bool(lib(mode).lnsb_backend_selected_by(device.encode(), value.encode() if value is not None else None))


def matches(node, token, mode="base"):
    return bool(lib(mode).lnsb_op_matches(ctypes.byref(node), token.encode()))


def disabled(node, disable, enable=None, mode="base"):
    return bool(lib(mode).lnsb_op_disabled_by(ctypes.byref(node), disable.encode() if disable is not None else None,
                                              enable.encode() if enable is not None else None))


def audit_line(backend, node, supported, reason, fmt=16, mode="base"):
    buf = ctypes.create_string_buffer(1024)
    lib(mode).lnsb_audit_line(backend.encode(), fmt, ctypes.byref(node), int(supported), reason.encode(), buf, 1024)
    return buf.value.decode()


def supports_op(device, node, fmt=16, mode="base"):
    return bool(lib(mode).lnsb_supports_op(device.encode(), fmt, ctypes.byref(node)))


def description(fmt=16, mode="base"):
    d = lib(mode).lnsb_device_description(fmt)
    return d.decode() if d else None


class Graph:
    """graph_compute over a list of node descriptors (a context per format
    and mode library: the stream, the weight cache and device scratch)"""

    def __init__(self, fmt=16, mode="base", cache_budget=-1, stream=None):
        self.lib = lib(mode)
        self.ctx = self.lib.lnsb_graph_ctx_create(fmt, cache_budget, stream)
        if not self.ctx:
            raise RuntimeError("lnsb_graph_ctx_create failed (no CUDA device, or the tables did not upload)")

    def compute(self, nodes):
        """runs the nodes in order; returns (status, index of the failing node or -1)"""
        arr = (ctypes.POINTER(Tensor) * len(nodes))(*[ctypes.pointer(n) for n in nodes])
        failed = ctypes.c_int(-1)
        st = self.lib.lnsb_graph_compute(self.ctx, arr, len(nodes), ctypes.byref(failed))
        return st, failed.value

    def close(self):
        if self.ctx:
            self.lib.lnsb_graph_ctx_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        self.close()
