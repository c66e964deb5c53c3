"""Runs packed_b200 on the reference-exported probe payload exactly as the
reference's runner invokes its native executable, and records the result.

    python tests/golden/record_packed_run.py OUTPUT_DIR

The reference's ``fhemamba.benchmarks.packed._run``
(src/fhemamba/benchmarks/packed.py:45-285) runs
``BINARY PAYLOAD/program.txt OUTPUT/native.json TOL TOL`` (tolerance 0.001,
no further flags at its defaults) and judges native.json and the exit code.
This script makes that call with packed_b200 on a B200 and writes
OUTPUT_DIR/native.json (the executable's own file) and
OUTPUT_DIR/recorded.json (argv tail, exit code).  Committed copies in
packed_probe_run/ let tests/test_reference_runner.py replay the run through
the reference's runner on a machine without a GPU.
"""
import json
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
TOLERANCE = "0.001"


def main(out: str) -> int:
    sys.path.insert(0, str(ROOT))
    from fhe_mamba_b200 import build
    build.build()
    out_dir = Path(out)
    out_dir.mkdir(parents=True, exist_ok=True)
    payload = HERE / "packed_probe"
    argv_tail = [TOLERANCE, TOLERANCE]
    cmd = [str(ROOT / "fhe_mamba_b200" / "packed_b200"), str(payload / "program.txt"),
           str(out_dir / "native.json")] + argv_tail
    rc = subprocess.run(cmd).returncode
    (out_dir / "recorded.json").write_text(json.dumps({"argv_tail": argv_tail, "returncode": rc}, indent=1) + "\n")
    return rc


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: record_packed_run.py OUTPUT_DIR")
    raise SystemExit(main(sys.argv[1]))
