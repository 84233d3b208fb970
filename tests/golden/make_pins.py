"""Regenerates tests/golden/reference_pins.json from the reference's committed
test outputs (results/sum32-evidence/*.txt of xlnsresearch/xlns-ggml-backend).

Those files are the only bit-level evidence of the reference's absent
arithmetic library (xlnscpp); every figure below is what the reference's own
deterministic test programs printed.  Run from the repo root with the
reference checkout available:

    python tests/golden/make_pins.py /path/to/reference
"""
import json
import os
import re
import sys


def floats(s):
    return [float(v) for v in re.findall(r"-?\d+\.\d+", s)]


def parse_standalone(text):
    out = {}
    m = re.search(r"two-term vs correctly-rounded \(n=(\d+)\): base max (\d+) ULP \(mean ([\d.]+)\), sum32 max (\d+) ULP \(mean ([\d.]+)\)", text)
    out["two_term"] = {"n": int(m.group(1)), "base_max": int(m.group(2)), "base_mean": float(m.group(3)),
                       "sum32_max": int(m.group(4)), "sum32_mean": float(m.group(5))}
    out["ones"] = {}
    for m in re.finditer(r"N=(\d+)\s+exact \d+\s+base\s+([\d.]+) \(\s*[\d.]+%\)\s+sum32\s+([\d.]+)", text):
        out["ones"][m.group(1)] = [float(m.group(2)), float(m.group(3))]
    out["long_dot"] = {}
    for m in re.finditer(r"K=(\d+)\s+mean rel err: base\s+([\d.]+)%\s+sum32\s+([\d.]+)%\s+\(sum32 better in (\d+)/64\)", text):
        out["long_dot"][m.group(1)] = [float(m.group(2)), float(m.group(3)), int(m.group(4))]
    out["rms_standalone"] = {}
    for m in re.finditer(r"n=(\d+)\s+max rel err: base\s+([\d.]+)%\s+sum32 ([\d.]+)%", text):
        out["rms_standalone"][m.group(1)] = [float(m.group(2)), float(m.group(3))]
    return out


def parse_suite(text):
    out = {}
    m = re.search(r"LNS mul mat \(4 x 3\):\s*\[([^\]]*)\]", text)
    out["mm4x3"] = floats(m.group(1))
    out["mm4x3_err"] = float(re.search(r"LNS mul mat max scaled error: ([\d.]+)%", text).group(1))
    m1 = re.search(r"max \|err\|/rms\(ref\): ([\d.]+)%\s+rms\(ref\): ([\d.]+)", text)
    m2 = re.search(r"LNS mul mat long NRMSE: ([\d.]+)%", text)
    out["mm_long"] = [float(m1.group(1)), float(m1.group(2)), float(m2.group(1))]
    out["softmax"] = [float(re.search(r"LNS softmax %s max abs error: ([\d.]+)" % c, text).group(1))
                      for c in ("short", "long", "scaled", "masked", "masked scaled")]
    out["rms_norm"] = [float(re.search(r"LNS rms_norm %s max scaled error: ([\d.]+)%%" % c, text).group(1))
                       for c in ("short", "576")]
    return out


def parse_swiglu(text, test_src):
    """The swiglu case of test-lns-backend.cpp (run_swiglu_test): its gate/up
    inputs from the test source, its printed 2 x 4 output from the log."""
    def arr(name):
        m = re.search(r"const float %s\[rows \* cols\] = \{([^}]*)\}" % name, test_src)
        return [float(v.rstrip("f")) for v in re.findall(r"-?\d+\.\d+f?", m.group(1))]
    m = re.search(r"LNS swiglu split \(4 x 2\):\s*\[([^\]]*)\]", text)
    return {"gate": arr("gate"), "up": arr("up"), "out": floats(m.group(1)),
            "source": "lns-backend/tests/test-lns-backend.cpp run_swiglu_test; unit-tests-lns16-base.txt"}


def parse_geglu_tanh(text, test_src):
    """The geglu case (run_geglu_test: the swiglu case's gate/up with gelu)
    and the tanh case (run_tanh_test: its 8 inputs from the test source)."""
    gg = re.search(r"LNS geglu split \(4 x 2\):\s*\[([^\]]*)\]", text)
    th = re.search(r"LNS tanh: \[([^\]]*)\]", text)
    m = re.search(r"static bool run_tanh_test.*?const float a\[n\] = \{([^}]*)\}", test_src, re.S)
    tin = [float(v.rstrip("f")) for v in re.findall(r"-?\d+\.\d+f?", m.group(1))]
    return {"geglu": floats(gg.group(1)), "tanh": floats(th.group(1)), "tanh_in": tin}


def main(ref):
    ev = os.path.join(ref, "results", "sum32-evidence")
    with open(os.path.join(ev, "standalone-sum32-invariants.txt")) as f:
        standalone = parse_standalone(f.read())
    suite = {}
    for name, fn in (("base", "unit-tests-lns16-base.txt"), ("monte", "unit-tests-lns16-monte.txt"),
                     ("lpvip", "unit-tests-lns16-lpvip.txt"), ("sum32", "unit-tests-lns16-sum32.txt"),
                     ("lns32", "unit-tests-lns32.txt")):
        with open(os.path.join(ev, fn)) as f:
            suite[name] = parse_suite(f.read())
    with open(os.path.join(ref, "lns-backend", "tests", "test-lns-backend.cpp")) as g:
        test_src = g.read()
    with open(os.path.join(ev, "unit-tests-lns16-base.txt")) as f:
        swiglu = parse_swiglu(f.read(), test_src)
    with open(os.path.join(ev, "unit-tests-lns32.txt")) as f:
        swiglu["out_lns32"] = parse_swiglu(f.read(), test_src)["out"]
    acts = {}
    for name, fn in (("lns16", "unit-tests-lns16-base.txt"), ("lns32", "unit-tests-lns32.txt")):
        with open(os.path.join(ev, fn)) as f:
            acts[name] = parse_geglu_tanh(f.read(), test_src)
    acts["source"] = ("lns-backend/tests/test-lns-backend.cpp run_geglu_test / run_tanh_test; "
                      "unit-tests-lns16-base.txt, unit-tests-lns32.txt")
    convert = {}
    with open(os.path.join(ref, "experiments", "dot-product-scaling", "results", "convert.jsonl")) as f:
        for line in f:
            if line.strip():
                rec = json.loads(line)
                convert[rec.pop("format")] = rec
    convert["source"] = ("experiments/dot-product-scaling/results/convert.jsonl "
                         "(protocol: experiments/dot-product-scaling/dot-bench.cpp convert())")
    # the synthetic dot-product records of the reference's CUDA backend
    # (dot-bench synth on LNSCUDA16 / LNSCUDA32), K <= 4096
    synth = []
    with open(os.path.join(ref, "experiments", "dot-product-scaling", "results", "synth.jsonl")) as f:
        for line in f:
            if line.strip():
                rec = json.loads(line)
                if rec["K"] <= 4096:
                    synth.append({k: rec[k] for k in ("config", "dist", "K", "acc", "acc_l2scale", "total")})
    pins = {
        "synth": {"records": synth,
                  "source": "experiments/dot-product-scaling/results/synth.jsonl (protocol: "
                            "experiments/dot-product-scaling/dot-bench.cpp synth(), run.py:62-75; "
                            "run on the reference's CUDA devices, run.py:46)"},
        "swiglu": swiglu,
        "source": "xlnsresearch/xlns-ggml-backend results/sum32-evidence/*.txt (outputs of "
                  "lns-backend/tests/test-lns16-sum32.cpp and test-lns-backend.cpp)",
        "standalone": standalone,
        "suite": suite,
        "lfsr": {"step7": 0xB403, "period": 65535},
        "convert": convert,
        "activations": acts,
    }
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_pins.json")
    with open(out, "w") as f:
        json.dump(pins, f, indent=1, sort_keys=True)
    print(out)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_pins.py <reference checkout>")
    main(sys.argv[1])
