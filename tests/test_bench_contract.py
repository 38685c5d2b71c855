"""bench.py's reference arm prints one JSON line with impl=reference and exits 0 (the driver runs it on
every box before the engine's own arm). Without a GPU (this test's setting) the single-GPU arm reports
why it could not run; with more than one GPU it reports that the reference's multi-GPU engine does not
build as shipped."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _line(*extra):
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", *extra], cwd=ROOT,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    return json.loads(lines[0])


def test_reference_arm_line():
    d = _line()
    assert d["impl"] == "reference" and d["unavailable"] and d["n_gpus"] == 1


def test_reference_arm_multi_gpu_line():
    d = _line("--gpus", "2")
    assert d["impl"] == "reference" and "does not build as shipped" in d["unavailable"] and d["n_gpus"] == 2
