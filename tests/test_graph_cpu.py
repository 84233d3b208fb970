"""The ggml backend's host layer (include/lnsb200_graph.h) on the CPU: the
op-support predicates and their audit reasons (lns-backend/common/
lns-op-support.h, lns-backend/cuda/lns-cuda-ops.cpp:25-230), backend
selection (lns-backend-config.h:55-136), op bisection (:138-199, checked
against lnsb200.policy), the LNS_OP_AUDIT line (:201-239), supports_op with
the environment, and the device description (ggml-lns-cuda.cpp:21-31)."""
import itertools
import json
import os
import subprocess
import sys

import numpy as np
import pytest

from lnsb200 import graph as G
from lnsb200 import policy

F = np.float32


def t(shape, type=None, name="", dtype=F, **kw):
    return G.tensor(np.zeros(shape, dtype), type=type, name=name, **kw)


def node(op, shape, src, params=(), name="", type=None, dtype=F):
    return G.tensor(np.zeros(shape, dtype), op=op, src=src, params=params, name=name, flags=G.FLAG_COMPUTE, type=type)


def test_names():
    lib = G.lib()
    assert lib.lnsb_op_name(G.OP["MUL_MAT"]) == b"MUL_MAT" and lib.lnsb_op_name(99) == b"UNKNOWN"
    u = node("UNARY", (4,), (t((4,)),), params=(G.UNARY["silu"],))
    g = node("GLU", (4,), (t((8,)),), params=(G.GLU["geglu"],))
    assert lib.lnsb_op_desc(u) == b"SILU" and lib.lnsb_op_desc(g) == b"GEGLU"


def test_mul_mat_predicate():
    w, x = t((4, 5)), t((3, 5))
    assert G.check(node("MUL_MAT", (3, 4), (w, x))) == (True, "lns_cuda_mul_mat")
    assert G.check(node("MUL_MAT", (3, 4), (t((4, 5), "f16", dtype=np.float16), x)))[0]
    assert G.check(node("MUL_MAT", (3, 4), (w, t((3, 5), "f16", dtype=np.float16)))) == \
        (False, "mul_mat_requires_src1_f32_and_convertible_src0")
    wt = np.zeros((5, 4), F).T                               # strided rows (a transposed view)
    assert G.check(node("MUL_MAT", (3, 4), (G.tensor(wt), x))) == (False, "mul_mat_requires_contiguous_rows")
    assert G.check(node("MUL_MAT", (3, 4), (w, x), type="f16", dtype=np.float16)) == \
        (False, "lns_cuda_mul_mat_requires_f32_dst")
    # broadcast: 2 weight slices against 4 activation slices; 3 against 4 is refused
    assert G.check(node("MUL_MAT", (4, 3, 4), (t((2, 4, 5)), t((4, 3, 5)))))[0]
    assert G.check(node("MUL_MAT", (4, 3, 4), (t((3, 4, 5)), t((4, 3, 5))))) == \
        (False, "lns_cuda_mul_mat_requires_whole_broadcast")
    # a quantised matrix: rows of whole blocks
    q = G.tensor(None, type="q8_0", ne=[64, 4, 1, 1], nb=[34, 68, 272, 272])
    assert G.check(node("MUL_MAT", (3, 4), (q, t((3, 64)))))[0]
    q.nb[1] = 80
    assert G.check(node("MUL_MAT", (3, 4), (q, t((3, 64))))) == (False, "lns_cuda_mul_mat_requires_packed_quantized_rows")


def test_elementwise_predicates():
    a = t((3, 8))
    assert G.check(node("ADD", (3, 8), (a, t((1, 8))))) == (True, "lns_cuda_binary")
    assert G.check(node("ADD", (3, 8), (a, t((1, 3))))) == (False, "lns_cuda_binary_requires_repeatable_src1")
    assert G.check(node("MUL", (3, 8), (a, t((1, 8), "f16", dtype=np.float16)))) == (False, "binary_requires_f32_srcs")
    assert G.check(node("MUL", (3, 4), (a, t((1, 8))))) == (False, "lns_cuda_requires_f32_dst_of_src0_shape")
    assert G.check(node("SCALE", (3, 8), (a,), params=(0.5, 0.0)))[0]
    assert G.check(node("SCALE", (8, 3), (G.tensor(np.zeros((8, 3), F).T.T.T),))) == \
        (False, "requires_contiguous_f32_src0_and_dst")
    for u in ("silu", "gelu", "relu", "tanh"):
        assert G.check(node("UNARY", (3, 8), (a,), params=(G.UNARY[u],))) == (True, "lns_cuda_unary")
    assert G.check(node("UNARY", (3, 8), (a,), params=(7,))) == (False, "unsupported_unary_op")
    assert G.check(node("RMS_NORM", (3, 8), (a,), params=(1e-5,)))[0]


def test_glu_predicate():
    g, u = t((3, 8)), t((3, 8))
    assert G.check(node("GLU", (3, 8), (g, u), params=(0,))) == (True, "glu_split_requires_matching_f32_contiguous_inputs")
    assert G.check(node("GLU", (3, 8), (g, t((3, 7))), params=(0,))) == (False, "glu_split_requires_matching_f32_contiguous_inputs")
    assert G.check(node("GLU", (3, 4), (t((3, 8)),), params=(1, 0)))[0]                 # fused [gate | up]
    assert G.check(node("GLU", (3, 4), (t((3, 9)),), params=(1, 0))) == (False, "glu_fused_requires_even_src0_and_half_width_dst")
    assert G.check(node("GLU", (3, 4), (t((3, 8)),), params=(5, 0))) == (False, "unsupported_glu_op")


def test_soft_max_and_rope_predicates():
    x = t((2, 4, 16))
    m = t((4, 32))                                       # a padded mask: wider rows are fine
    assert G.check(node("SOFT_MAX", (2, 4, 16), (x, m), params=(0.125, 0.0))) == (True, "soft_max_f32")
    assert G.check(node("SOFT_MAX", (2, 4, 16), (x, t((4, 8))), params=(0.125, 0.0))) == \
        (False, "lns_cuda_soft_max_mask_smaller_than_src0")
    assert G.check(node("SOFT_MAX", (2, 4, 16), (x, m), params=(0.125, 8.0))) == (False, "soft_max_alibi_unsupported")
    sinks = node("SOFT_MAX", (2, 4, 16), (x, m, t((2,))), params=(1.0, 0.0))
    assert G.check(sinks) == (False, "soft_max_sinks_unsupported")
    q = t((1, 5, 9, 64))                                 # [tokens 5][heads 9][dim 64]: ne2 = positions
    pos = t((5,), "i32", dtype=np.int32)
    rp = lambda mode, ext=0.0, nd=64, src=(q, pos): node("ROPE", (1, 5, 9, 64), src,      # noqa: E731
                                                         params=(0, nd, mode, 0, 0, 1e5, 1.0, ext, 1.0))
    assert G.check(rp(0)) == (True, "lns_cuda_rope") and G.check(rp(G.ROPE_NEOX))[0]
    assert G.check(rp(8)) == (False, "rope_mode_unsupported")
    assert G.check(rp(0, ext=1.0)) == (False, "rope_scaling_unsupported")
    assert G.check(rp(0, nd=63)) == (False, "lns_cuda_rope_requires_even_n_dims")
    assert G.check(rp(0, src=(q, t((5,))))) == (False, "lns_cuda_rope_requires_i32_positions")


def test_views_and_unsupported_ops():
    a = t((3, 8))
    for op in ("NONE", "RESHAPE", "VIEW", "PERMUTE", "TRANSPOSE"):
        assert G.check(node(op, (3, 8), (a,))) == (True, "supported_view_or_noop")
    for op in ("GET_ROWS", "CPY", "CONT"):
        assert G.check(node(op, (3, 8), (a,))) == (False, "unsupported_op")


def test_backend_selection():
    assert G.resolve_selection(None) == ["LNS16"] and G.resolve_selection("") == ["LNS16"]
    assert G.resolve_selection("cuda") == ["LNSCUDA16", "LNS16"]
    assert G.resolve_selection("CUDA32") == ["LNSCUDA32", "LNS32"]
    assert G.resolve_selection(" lnscuda16 , 32") == ["lnscuda16", "LNS32"]
    assert G.resolve_selection("bogus") == ["LNS16"]                    # nothing valid: the default
    assert G.selected("LNSCUDA16", "cuda") and G.selected("lns16", "cuda")
    assert not G.selected("LNSCUDA16", None) and not G.selected("LNSCUDA32", "cuda16")
    assert G.selected("LNSCUDA16", "LNSCUDA16") and not G.selected("LNS16", "LNSCUDA16")


def test_bisection_matches_the_python_policy():
    """LNS_DISABLE_OPS / LNS_ENABLE_OPS in C++ agree with lnsb200.policy.op_disabled"""
    ops = ["MUL_MAT", "SOFT_MAX", "RMS_NORM", "ADD"]
    names = ["ffn_down-3", "kq-12", "kqv_out-5", "result_output", ""]
    src1s = ["kqv_out-2", "attn_norm-1", ""]
    lists = [None, "", "MUL_MAT", "soft_max", "ffn_down", "MUL_MAT:kq-*", "*-5", "MUL_MAT:<kqv_out-*",
             "rms_norm, result_output", "kq-1[0-9]", "RMS_NORM:ffn"]
    n = 0
    for op, name, s1, dis, en in itertools.product(ops, names, src1s, lists[1:], lists):
        b = t((2, 4), name=s1)
        nd = node(op, (2, 4), (t((2, 4)), b), name=name)
        env = {"LNS_DISABLE_OPS": dis}
        if en is not None:
            env["LNS_ENABLE_OPS"] = en
        want = policy.op_disabled(op, name, s1 or None, env=env)
        assert G.disabled(nd, dis, en) == want, (op, name, s1, dis, en)
        n += 1
    assert n > 1000
    # the op's desc counts too (UNARY ops by their unary name)
    u = node("UNARY", (4,), (t((4,)),), params=(G.UNARY["gelu"],), name="ffn_gelu-0")
    assert G.matches(u, "gelu") and G.matches(u, "UNARY") and G.matches(u, "GELU:ffn") and not G.matches(u, "SILU")


def test_audit_line():
    x = t((2, 4, 16), name="kq-3")
    nd = node("SOFT_MAX", (2, 4, 16), (x, t((4, 16))), params=(1.0, 0.0), name="kq_soft_max-3")
    d = json.loads(G.audit_line("LNSCUDA16", nd, True, "soft_max_f32"))
    assert d == {"event": "lns_supports_op", "backend": "LNSCUDA16", "sum_mode": "base", "op": "SOFT_MAX",
                 "desc": "SOFT_MAX", "supported": True, "dst_type": "f32", "src_types": ["f32", "f32", "null", "null"],
                 "shape": [16, 4, 2, 1], "reason": "soft_max_f32"}
    d32 = json.loads(G.audit_line("LNSCUDA32", nd, False, "x", fmt=32))
    assert "sum_mode" not in d32 and d32["supported"] is False


@pytest.mark.parametrize("mode,desc", [("base", "xlns16, sum=base"), ("monte", "xlns16, sum=monte, monte=pure16"),
                                       ("monte_bylpvip", "xlns16, sum=monte, monte=bylpvip"),
                                       ("lpvip", "xlns16, sum=lpvip"), ("sum32", "xlns16, sum=sum32")])
def test_description(mode, desc):
    d = G.description(16, mode)
    assert d.startswith("Logarithmic Number System on CUDA (%s)" % desc)
    assert G.description(32, mode).startswith("Logarithmic Number System on CUDA (xlns32)")


PROBE = r"""
import sys
sys.path.insert(0, {pkg!r})
import numpy as np
from lnsb200 import graph as G
w, x = G.tensor(np.zeros((4, 5), np.float32)), G.tensor(np.zeros((3, 5), np.float32), name="attn_norm-0")
mm = G.tensor(np.zeros((3, 4), np.float32), op="MUL_MAT", src=(w, x), name="ffn_down-0", flags=1)
sm = G.tensor(np.zeros((3, 5), np.float32), op="SOFT_MAX", src=(x,), params=(1.0, 0.0), name="kq_soft_max-0", flags=1)
print(int(G.supports_op("LNSCUDA16", mm)), int(G.supports_op("LNSCUDA16", sm)), int(G.supports_op("LNSCUDA32", sm, fmt=32)))
"""


@pytest.mark.parametrize("env,want", [
    ({}, "0 0 0"),                                                  # default selection: LNS16 only
    ({"GGML_LNS_BACKEND": "cuda"}, "1 1 0"),
    ({"GGML_LNS_BACKEND": "cuda,cuda32"}, "1 1 1"),
    ({"GGML_LNS_BACKEND": "cuda", "LNS_DISABLE_OPS": "ffn_down"}, "0 1 0"),
    ({"GGML_LNS_BACKEND": "cuda", "LNS_ENABLE_OPS": "SOFT_MAX"}, "0 1 0"),
    ({"GGML_LNS_BACKEND": "cuda", "LNS_ENABLE_OPS": ""}, "0 0 0"),
])
def test_supports_op_reads_the_environment(env, want):
    from conftest import PKG
    e = {k: v for k, v in os.environ.items() if k not in ("GGML_LNS_BACKEND", "LNS_DISABLE_OPS", "LNS_ENABLE_OPS",
                                                             "LNS_OP_AUDIT")}
    e.update(env)
    e["LNS_OP_AUDIT"] = "1"
    r = subprocess.run([sys.executable, "-c", PROBE.format(pkg=PKG)], env=e, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert r.stdout.split("\n")[0].strip() == want
    audits = [json.loads(line) for line in r.stderr.splitlines() if line.startswith("{")]
    assert len(audits) == 3                                          # one line per query
    if "GGML_LNS_BACKEND" not in env:
        assert all(a["reason"] == "disabled_by_env" for a in audits)
    else:
        assert audits[0]["reason"] == "lns_cuda_mul_mat" and audits[0]["backend"] == "LNSCUDA16"


def test_graph_context_needs_a_device():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(RuntimeError):
        G.Graph(16)
