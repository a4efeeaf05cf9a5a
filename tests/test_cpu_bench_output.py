"""bench.py's output contract: rank 0's stdout holds exactly one JSON line, even when a library
(NCCL prints its version line at communicator set-up) writes to file descriptor 1."""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent

CHILD = r"""
import os, sys
sys.path.insert(0, sys.argv[1])
import bench
bench.quiet_stdout()
os.write(1, b"NCCL version 0.0.0 (a library writing to fd 1)\n")
print("a stray print")
bench.emit({"metric": "decode tok/s", "value": 1.0})
"""


def test_stdout_holds_only_the_json_line():
    r = subprocess.run([sys.executable, "-c", CHILD, str(ROOT)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    lines = r.stdout.splitlines()
    assert len(lines) == 1, r.stdout
    assert json.loads(lines[0]) == {"metric": "decode tok/s", "value": 1.0}
    assert "NCCL version" in r.stderr and "a stray print" in r.stderr


def test_reference_arm_without_a_cpu_path_prints_its_unavailable_line():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--workload", "residual", "--impl", "reference"],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    lines = r.stdout.splitlines()
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and "unavailable" in d
