"""bench.py's reference arm prints its one-line `unavailable` JSON and exits 0."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_unavailable_line():
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--gpus", "1"], cwd=ROOT,
                         capture_output=True, text=True, timeout=120)
    assert out.returncode == 0
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and "unavailable" in line
