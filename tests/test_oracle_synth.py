"""The oracle's mul_mat against the reference CUDA backend's synthetic
dot-product records.

oracle/synthstat.cpp replays experiments/dot-product-scaling/dot-bench.cpp
synth() (run.py:62-75: seed 1, 1024 weight rows x 4 tokens, normal weights;
signed, positive and softmax ("attn") activations) through the oracle's
mul_mat and prints the reference's error statistics; tests/golden/
reference_pins.json holds the records the reference's run printed for K <= 4096
(tests/golden/make_pins.py).  A record is reproduced when all fifteen figures
(bias, sd, rms, mean_abs, rel_l2 of the three error measures) agree to the six
significant digits the reference prints.

SYNTH_PINNED is every record reproduced: the whole base configuration (the
xlns16 adder, the conversions, the reduction order, the output decode) and
six sum32 records (signed K = 16, 32; softmax-weighted K = 16, 32, 64;
positive K = 64).  The other sum32 "positive" records need a rounded sb
interpolation, which the reference's CPU library -- the parity target --
does not use (its sums of ones and LNS32 rms_norm printouts need the floored
one); the mixed-sign records beyond K = 64 differ in the fifth digit (db above
one octave).  They are printed beside the reference's by test_synth_report.
"""
import json
import os

import pytest

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "reference_pins.json")
KS = (16, 32, 64, 128, 256, 512, 1024, 2048, 4096)
SYNTH_PINNED = ([("base", d, k) for d in ("signed", "positive", "attn") for k in KS] +
                [("sum32", "signed", 16), ("sum32", "signed", 32), ("sum32", "attn", 16), ("sum32", "attn", 32),
                 ("sum32", "attn", 64), ("sum32", "positive", 64)])
FIELDS = ("bias", "sd", "rms", "mean_abs", "rel_l2")


def _records():
    with open(GOLDEN) as f:
        return {(r["config"], r["dist"], r["K"]): r for r in json.load(f)["synth"]["records"]}


def _digits(rec):
    return {(m, k): "%.6g" % rec[m][k] for m in ("acc", "acc_l2scale", "total") for k in FIELDS}


@pytest.mark.parametrize("key", SYNTH_PINNED, ids=lambda k: "%s-%s-%d" % k)
def test_synth_record(orc, key):
    want = _records()[key]
    got = orc.synthstat(*key)
    assert _digits(got) == _digits(want)


def test_synth_report(orc, capsys):
    """Prints the acc rms and bias of every other record beside the
    reference's (informational; K <= 256 to keep the suite short)."""
    recs = _records()
    rows = []
    for key, want in sorted(recs.items()):
        if key in SYNTH_PINNED or key[2] > 256:
            continue
        got = orc.synthstat(*key)
        rows.append("%-14s %-9s K=%-4d rms %.6g / %.6g  bias %.6g / %.6g  %s" % (
            key[0], key[1], key[2], got["acc"]["rms"], want["acc"]["rms"], got["acc"]["bias"], want["acc"]["bias"],
            "same" if _digits(got) == _digits(want) else "differs"))
    with capsys.disabled():
        print("\nsynthetic record            this oracle / reference")
        print("\n".join(rows))
