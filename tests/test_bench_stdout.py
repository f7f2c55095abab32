"""bench.py under torchrun: whatever a library writes to the process's stdout
(NCCL prints its version banner there) goes to stderr, and the JSON line is
the only thing on stdout.  Runs on the CPU: a child process stands in for a
rank, with a C-level write in place of the banner."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import os, sys
sys.path.insert(0, sys.argv[1])
import bench
print("before the process group", flush=True)   # ordinary output before redirection stays
bench.quiet_stdout()
os.write(1, b"NCCL version x.y.z\n")            # a library banner on fd 1
print("a stray print", flush=True)
bench.emit({"metric": "m", "value": 1.0})
"""


def test_emit_keeps_stdout_to_the_json_line():
    r = subprocess.run([sys.executable, "-c", CHILD, ROOT], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    out = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert out[0] == "before the process group"
    assert json.loads(out[-1]) == {"metric": "m", "value": 1.0}
    assert len(out) == 2
    assert "NCCL version x.y.z" in r.stderr and "a stray print" in r.stderr
