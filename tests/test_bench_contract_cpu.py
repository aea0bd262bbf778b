"""bench.py's command-line contract, checked without a GPU.

The reference arm has no runnable build here (a C#/.NET project, no dotnet on the image), so
``--impl reference`` must print one JSON line with ``impl`` and ``unavailable`` and exit 0; the default
arguments are one GPU and a short run with at least three warm-up steps.
"""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_reports_unavailable_and_exits_zero():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--gpus", "1",
                          "--steps", "2", "--warmup", "3"], capture_output=True, text=True, timeout=120, cwd=ROOT)
    assert out.returncode == 0, out.stderr
    lines = [l for l in out.stdout.splitlines() if l.strip()]
    assert len(lines) == 1
    rec = json.loads(lines[0])
    assert rec["impl"] == "reference" and rec["unavailable"]


def test_default_arguments_are_one_gpu_and_a_short_run(monkeypatch):
    sys.path.insert(0, ROOT)
    import bench
    monkeypatch.setattr(sys, "argv", ["bench.py"])
    a = bench.parse()
    assert a.gpus == 1 and a.impl == "ours" and a.workload == "decoder"
    assert 1 <= a.steps <= 100 and a.warmup >= 3
