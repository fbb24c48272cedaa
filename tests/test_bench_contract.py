"""The bench.py command-line contract that runs without a GPU."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_unavailable_line():
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--gpus", "1", "--steps", "3",
                          "--warmup", "3"], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unavailable"]


def test_bench_defaults_and_engine_choices():
    import bench  # noqa: F401 - module imports without touching CUDA

    src = open(os.path.join(ROOT, "bench.py")).read()
    assert '"--engine", default="tma"' in src and '"--layer-batch", type=int, default=8' in src
    assert '"--steps", type=int, default=3' in src and '"--warmup", type=int, default=3' in src
