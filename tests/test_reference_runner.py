"""The reference's own packed runner judges packed_b200.

The committed payload was exported by the reference's exporter
(golden/make_packed_probe.py: one synthetic Mamba-3 SISO mixer, 2 steps), and
packed_b200's native.json and exit code on a B200 were recorded by
golden/record_packed_run.py, invoked as the runner invokes its executable.
Here a stand-in executable checks that the runner passes exactly that argv
(PROGRAM RESULT POLY_TOL EXACT_TOL) and writes the recorded native.json; the
runner's gates (src/fhemamba/benchmarks/packed.py:151-272: schema, encrypted,
passed, one error per manifest output, finite errors within the tolerance,
exit code 0) must accept it.  Needs the reference's source next to this
checkout (or FHEMAMBA_REFERENCE_SRC); skipped where it is absent.  No GPU.
"""
import json
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = ROOT / "tests" / "golden"


def _reference_src():
    cands = [Path(os.environ["FHEMAMBA_REFERENCE_SRC"])] if os.environ.get("FHEMAMBA_REFERENCE_SRC") else []
    cands.append(ROOT.parent / "reference" / "src")
    for c in cands:
        if (c / "fhemamba" / "benchmarks" / "packed.py").exists():
            return c
    return None


def _replay(tmp_path, native_path, returncode, argv_tail):
    """A stand-in executable that checks its argv and writes native_path."""
    shim = tmp_path / "packed_b200_replay"
    shim.write_text(
        f"#!{sys.executable}\n"
        "import shutil, sys\n"
        "args = sys.argv[1:]\n"
        f"assert len(args) == 4 and args[0].endswith('program.txt') and args[1].endswith('native.json') "
        f"and args[2:] == {argv_tail!r}, args\n"
        f"shutil.copyfile({str(native_path)!r}, args[1])\n"
        f"sys.exit({int(returncode)})\n")
    shim.chmod(0o755)
    return shim


def _runner():
    src = _reference_src()
    if src is None:
        pytest.skip("the reference's source is not next to this checkout")
    sys.path.insert(0, str(src))
    from fhemamba.benchmarks.packed import _run
    return _run


def test_reference_runner_accepts_recorded_packed_b200_run(tmp_path):
    _run = _runner()
    rec_dir = GOLDEN / "packed_probe_run"
    rec = json.loads((rec_dir / "recorded.json").read_text())
    shim = _replay(tmp_path, rec_dir / "native.json", rec["returncode"], rec["argv_tail"])
    record = _run(shim, GOLDEN / "packed_probe", tmp_path / "out")
    assert record["returncode"] == 0 and record["passed"] is True, record
    native = json.loads((rec_dir / "native.json").read_text())
    manifest = json.loads((GOLDEN / "packed_probe" / "manifest.json").read_text())
    assert native["schema"] == "fhemamba-packed-result-v1" and native["encrypted"] is True
    assert len(native["per_output_errors"]) == len(manifest["output_names"])


def test_reference_runner_rejects_a_planted_error(tmp_path):
    """A mistake planted in a copy of the recorded result (one output's error
    above the runner's tolerance) makes the same runner fail the run, so the
    acceptance above is the runner's judgement, not a formality."""
    _run = _runner()
    rec_dir = GOLDEN / "packed_probe_run"
    rec = json.loads((rec_dir / "recorded.json").read_text())
    native = json.loads((rec_dir / "native.json").read_text())
    native["max_abs_error_vs_polynomial"] = 0.5
    bad = tmp_path / "native_bad.json"
    bad.write_text(json.dumps(native))
    shim = _replay(tmp_path, bad, rec["returncode"], rec["argv_tail"])
    record = _run(shim, GOLDEN / "packed_probe", tmp_path / "out")
    assert record["passed"] is False
