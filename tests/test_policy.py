"""LNS16_SUM_POLICY parsing and op matching (lnsb200.policy) against the
reference's token rules (lns-backend/common/lns-backend-config.h:33-49,
141-175; the examples of its SETUP.md:290-300)."""
import pytest

from lnsb200.policy import SumPolicy, name_matches, op_matches, split_list


def test_split_list():
    assert split_list(" a, b ,,c ,") == ["a", "b", "c"]
    assert split_list("") == []


def test_name_matches():
    assert name_matches("ffn_down-12", "ffn_down")           # substring, case-sensitive
    assert not name_matches("ffn_down-12", "FFN_DOWN")
    assert name_matches("kq-5", "*-5") and not name_matches("kq-15", "*-5")   # wildcard: the whole name
    assert name_matches("kq-3", "kq-[0-4]")
    assert not name_matches("", "kq") and not name_matches(None, "kq")


def test_op_matches():
    assert op_matches("soft_max", "SOFT_MAX", "kq_soft_max-0")
    assert op_matches("MUL_MAT:kq-*", "MUL_MAT", "kq-3")
    assert not op_matches("MUL_MAT:kq-*", "SOFT_MAX", "kq-3")
    assert not op_matches("MUL_MAT:kq-*", "MUL_MAT", "kqv-3")
    assert op_matches("MUL_MAT:<kqv_out-*", "MUL_MAT", "attn_out-2", "kqv_out-2")
    assert not op_matches("MUL_MAT:<kqv_out-*", "MUL_MAT", "kqv_out-2", "kqv-2")
    assert op_matches("result_output", "MUL_MAT", "result_output")


def test_policy_first_rule_wins_and_default():
    p = SumPolicy("MUL_MAT:kqv-*=sum32, SOFT_MAX=lpvip, MUL_MAT=monte", default="base")
    assert p.mode_for("MUL_MAT", "kqv-4") == "sum32"
    assert p.mode_for("MUL_MAT", "Qcur-4") == "monte"
    assert p.mode_for("SOFT_MAX", "kq_soft_max-4") == "lpvip"
    assert p.mode_for("RMS_NORM", "norm-4") == "base"
    assert p.mode_for("ADD", "ffn_out-4") == "base"            # not a reduction: always the default
    assert p.modes() == ["base", "lpvip", "monte", "sum32"]


def test_policy_errors():
    with pytest.raises(ValueError):
        SumPolicy("MUL_MAT")
    with pytest.raises(ValueError):
        SumPolicy("MUL_MAT=fast")
    with pytest.raises(ValueError):
        SumPolicy(None, default="exact")


def test_policy_from_env(monkeypatch):
    monkeypatch.setenv("LNS16_SUM_POLICY", "RMS_NORM=sum32")
    assert SumPolicy.from_env("base").mode_for("RMS_NORM", "norm-0") == "sum32"
    monkeypatch.delenv("LNS16_SUM_POLICY")
    assert SumPolicy.from_env("lpvip").rules == []


TINY = dict(n_layer=2, n_embd=64, n_head=4, n_head_kv=2, head_dim=16, n_ff=128, vocab=300, rope_base=10000.0, eps=1e-5)


def _logits(policy, mode="base"):
    from lnsb200 import model
    from oracle_model import OracleOps
    w = model.init_weights(TINY, seed=2)
    o = OracleOps(TINY, w, mode=mode, n_ctx=16, policy=policy)
    return model.forward(o, TINY, model.prompt_ids(TINY, 5, seed=2), 0)


def test_model_policy_reaches_the_ops():
    """on the CPU oracle: a rule naming the default mode changes nothing; a rule
    with another mode changes the logits only through the ops it selects"""
    import numpy as np
    base = _logits(None)
    assert np.array_equal(base, _logits("MUL_MAT=base,SOFT_MAX=base"))
    assert not np.array_equal(base, _logits("MUL_MAT:kqv-*=sum32"))
    assert not np.array_equal(base, _logits("RMS_NORM=lpvip"))
    assert np.array_equal(base, _logits("MUL_MAT:nothing-*=sum32"))


def test_op_bisection():
    from lnsb200.policy import op_disabled
    assert not op_disabled("MUL_MAT", "ffn_down-3", env={})
    assert op_disabled("MUL_MAT", "ffn_down-3", env={"LNS_DISABLE_OPS": "MUL_MAT,ffn_down"})
    assert op_disabled("ADD", "ffn_down-3", env={"LNS_DISABLE_OPS": "ffn_down"})          # substring of the name
    assert not op_disabled("ADD", "ffn_out-3", env={"LNS_DISABLE_OPS": "ffn_down"})
    assert op_disabled("SOFT_MAX", "kq_soft_max-0", env={"LNS_ENABLE_OPS": "MUL_MAT"})  # only matching ops run in LNS
    assert not op_disabled("MUL_MAT", "kq-0", env={"LNS_ENABLE_OPS": "MUL_MAT"})
    assert op_disabled("MUL_MAT", "kq-0", env={"LNS_ENABLE_OPS": ""})                   # set but empty: none
    assert op_disabled("MUL_MAT", "kq-0", env={"LNS_ENABLE_OPS": "MUL_MAT", "LNS_DISABLE_OPS": "kq-*"})
