"""bench.py's output contract, on CPU: stdout carries exactly one JSON line
(library banners such as NCCL's version line, written to file descriptor 1,
go to stderr), and the metric is BASELINE.json's."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_stdout_is_the_json_line_alone():
    code = (
        "import os, sys; sys.path.insert(0, %r); import bench; bench.json_stdout(); "
        "os.write(1, b'NCCL version x.y\\n'); print('a python print'); bench.emit({'metric': 'm', 'value': 1})"
        % ROOT)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    lines = r.stdout.splitlines()
    assert len(lines) == 1 and json.loads(lines[0]) == {"metric": "m", "value": 1}
    assert "NCCL version" in r.stderr and "a python print" in r.stderr


def test_metric_is_baselines():
    sys.path.insert(0, ROOT)
    import bench
    with open(os.path.join(ROOT, "BASELINE.json")) as f:
        assert json.load(f)["metric"] == bench.METRIC
