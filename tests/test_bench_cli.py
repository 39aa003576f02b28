"""The benchmark's reference arm on the host (no GPU): one JSON line with the
contract's keys for the default workload, an `unavailable` line for the
others, exit status 0 in both cases."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(*args):
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    return json.loads(r.stdout.strip().splitlines()[-1])


def test_reference_arm_line():
    d = _run("--impl", "reference", "--grid", "64", "--steps", "3", "--warmup", "1")
    assert d["impl"] == "reference" and d["steps"] == 3 and d["warmup"] == 1
    for k in ("metric", "value", "unit", "n_gpus", "ms_per_step", "higher_is_better", "scaling",
              "dtype", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["config"]["n"] == 64 * 64


def test_reference_arm_other_workloads_unavailable():
    d = _run("--impl", "reference", "--workload", "scan")
    assert d["impl"] == "reference" and "unavailable" in d
