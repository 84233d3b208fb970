"""A summation mode per op: LNS16_SUM_POLICY (lns-backend/cuda/lns-cuda-context.cpp:
221-269; token syntax lns-backend/common/lns-backend-config.h:33-49, 141-175;
described in SETUP.md:290-300 of the reference).

The spec is a comma-separated list of `selector=mode` rules; the first rule
whose selector matches an op picks the mode of that op's reductions
(MUL_MAT, MUL_MAT_ID, SOFT_MAX, RMS_NORM), every other op keeps the default
mode.  A selector matches

  * the op name, case-insensitively (`SOFT_MAX`);
  * `OP:pattern`: that op whose tensor name matches the pattern
    (`MUL_MAT:kq-*`), or whose second input's name matches when the pattern
    starts with `<` (`MUL_MAT:<kqv_out-*`);
  * `pattern` alone: any op whose tensor name matches it.

A pattern with any of `*?[` is a case-sensitive wildcard over the whole name
(`*-5` is layer 5 only); otherwise it is a case-sensitive substring.

Every summation mode is its own library here (liblnsb200_<mode>.so), so every
mode can serve a rule -- the reference needs a GGML_LNSCUDA16_MIXED build for
base, lpvip and sum32 and serves monte only as the build's own mode.  A rule
that is not `selector=mode`, or names an unknown mode, raises ValueError
where the reference aborts.
"""
import fnmatch
import os

from ._lib import MODES

REDUCTION_OPS = ("MUL_MAT", "MUL_MAT_ID", "SOFT_MAX", "RMS_NORM")


def split_list(spec):
    """comma-separated tokens, blanks trimmed, empty tokens dropped"""
    return [t.strip(" \t") for t in spec.split(",") if t.strip(" \t")]


def name_matches(name, pattern):
    if not name:
        return False
    if any(c in pattern for c in "*?["):
        return fnmatch.fnmatchcase(name, pattern)
    return pattern in name


def op_matches(tok, op, name, src1_name=None):
    """op: the ggml op name (e.g. MUL_MAT); name: the op's tensor name;
    src1_name: the name of its second input"""
    if tok.lower() == op.lower():
        return True
    pattern = tok
    if ":" in tok:
        want, pattern = tok.split(":", 1)
        if want.lower() != op.lower():
            return False
    if pattern.startswith("<"):
        return name_matches(src1_name, pattern[1:])
    return name_matches(name, pattern)


class SumPolicy:
    def __init__(self, spec=None, default="base"):
        if default not in MODES:
            raise ValueError("unknown summation mode %r" % default)
        self.default = default
        self.rules = []
        for rule in split_list(spec or ""):
            eq = rule.rfind("=")
            if eq < 0:
                raise ValueError("LNS16_SUM_POLICY rule %r is not selector=mode" % rule)
            mode = rule[eq + 1:].strip()
            if mode not in MODES:
                raise ValueError("LNS16_SUM_POLICY mode %r is not one of %s" % (mode, ", ".join(MODES)))
            self.rules.append((rule[:eq], mode))

    @classmethod
    def from_env(cls, default="base", env="LNS16_SUM_POLICY"):
        return cls(os.environ.get(env), default)

    def mode_for(self, op, name, src1_name=None):
        if op.upper() in REDUCTION_OPS:
            for sel, mode in self.rules:
                if op_matches(sel, op, name, src1_name):
                    return mode
        return self.default

    def modes(self):
        return sorted({self.default} | {m for _, m in self.rules})


def op_disabled(op, name, src1_name=None, env=None):
    """LNS_DISABLE_OPS / LNS_ENABLE_OPS op bisection (lns-backend/common/
    lns-backend-config.h:186-199): with LNS_ENABLE_OPS set, an op runs in LNS
    only if a token of it matches (set but empty: no op does); an op matching
    a token of LNS_DISABLE_OPS falls back.  Same token syntax as the sum
    policy's selectors.  True means "not in LNS"."""
    env = os.environ if env is None else env
    if "LNS_ENABLE_OPS" in env:
        if not any(op_matches(t, op, name, src1_name) for t in split_list(env["LNS_ENABLE_OPS"])):
            return True
    return any(op_matches(t, op, name, src1_name) for t in split_list(env.get("LNS_DISABLE_OPS", "")))
