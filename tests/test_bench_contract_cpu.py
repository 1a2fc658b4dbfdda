"""The benchmark driver contract on CPU: the reference arm prints exactly one JSON line with
``impl`` and ``unavailable`` and exits 0, and the arguments the driver passes parse."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_unavailable_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--gpus", "1",
                        "--steps", "3", "--warmup", "3"], cwd=ROOT, capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unavailable"]


def test_driver_arguments_parse():
    sys.path.insert(0, ROOT)
    import bench
    old = sys.argv
    try:
        for argv in (["bench.py"], ["bench.py", "--gpus", "8", "--steps", "20", "--warmup", "3"],
                     ["bench.py", "--impl", "ref-algorithm", "--ref-requests", "1"],
                     ["bench.py", "--config", "awq-h2o", "--comm", "nccl"]):
            sys.argv = argv
            a = bench.parse()
            assert a.steps > 0 and a.warmup >= 0 and a.gpus >= 1
    finally:
        sys.argv = old
