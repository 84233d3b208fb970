"""bench.py's reference arm (`--impl reference`) runs on the host alone: the
reference's CPU algorithm (this repository's restatement under oracle/) timed
on a bounded sample of the bench workload.  Its one JSON line carries the
keys the benchmark contract asks of it, with the same metric and unit as the
GPU arm."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_json_line():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "0"], capture_output=True, text=True, timeout=300,
                       env=dict(os.environ, RANK="0", WORLD_SIZE="1"))
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == "LNS16 mul_mat G-LNSadd/s" and d["unit"] == "G-LNSadd/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 1
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["config"]["mode"] == "base"


def test_reference_arm_other_ranks_exit_quietly():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "0"], capture_output=True, text=True, timeout=120,
                       env=dict(os.environ, RANK="1", WORLD_SIZE="2"))
    assert r.returncode == 0 and not [l for l in r.stdout.splitlines() if l.startswith("{")]
