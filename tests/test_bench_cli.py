"""The benchmark's reference arm on the host (no GPU): one JSON line with the
contract's keys for the default workload and for the others, the `workloads`
object beside the headline, exit status 0."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(*args):
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    return json.loads(r.stdout.strip().splitlines()[-1])


def _contract(d):
    for k in ("metric", "value", "unit", "n_gpus", "ms_per_step", "higher_is_better", "scaling",
              "dtype", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0


def test_reference_arm_line():
    d = _run("--impl", "reference", "--grid", "64", "--steps", "3", "--warmup", "1",
             "--extra", "none")
    assert d["impl"] == "reference" and d["steps"] == 3 and d["warmup"] == 1
    _contract(d)
    assert d["config"]["n"] == 64 * 64 and "workloads" not in d


def test_reference_arm_other_workloads():
    for w in ("scan", "spmv1"):
        d = _run("--impl", "reference", "--workload", w, "--steps", "2", "--warmup", "1")
        assert d["impl"] == "reference" and d["value"] > 0
        _contract(d)


def test_reference_arm_workloads_object(monkeypatch, capsys):
    """The default run carries a `workloads` object keyed by configuration,
    each entry with the same fields (here with only the scan, to stay fast)."""
    sys.path.insert(0, ROOT)
    import bench
    monkeypatch.setattr(bench, "EXTRA", ["scan"])
    bench.main(["--impl", "reference", "--grid", "64", "--steps", "2", "--warmup", "1"])
    d = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    _contract(d)
    w = d["workloads"]["scan"]
    assert w["unit"] == "Gcounts/s" and w["value"] > 0 and w["cpu_baseline"]["cores"] == 1
    assert w["e2e"]["value"] == w["value"]
