"""The packed-program executor on the GPU, through the packed_b200 drop-in
executable (same argv, exit codes and result JSON as the reference's
packed_fideslib) and through the in-process C-ABI call.

Fixtures were compiled by the reference's own PackedProgram
(tests/golden/make_programs.py); each carries the reference's polynomial and
exact output values, which the decrypted outputs must match.
"""
import json
import os
import subprocess

import pytest

from fhe_mamba_b200.program import CLI, run_program

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _run_cli(tmp_path, name, poly_tol, exact_tol, *flags):
    out = tmp_path / "native.json"
    r = subprocess.run([CLI, os.path.join(GOLDEN, name), str(out), str(poly_tol), str(exact_tol), "--ring-log", "12",
                        *flags], capture_output=True, text=True, timeout=600)
    report = json.loads(out.read_text()) if out.exists() else None
    return r, report


def test_all_operations(tmp_path):
    r, rep = _run_cli(tmp_path, "packed_all_ops_v2.txt", 1e-6, 5e-2, "--hoist-rotations")
    assert r.returncode == 0, r.stderr
    assert rep["schema"] == "fhemamba-packed-result-v1" and rep["encrypted"] and rep["passed"]
    assert rep["max_abs_error_vs_polynomial"] < 1e-6 and rep["non_finite"] == 0
    assert rep["bootstraps"] == 0 and rep["ct_ct_mul"] == 2
    assert set(rep["operation_stats"]) == {"input", "linear", "linear_ref", "add", "mul", "mulp", "addp", "cheb",
                                           "sum", "repeat", "gather", "public", "scatter"}


def test_wide_linear_and_gather(tmp_path):
    r, rep = _run_cli(tmp_path, "packed_linear_v2.txt", 1e-6, 1e-6)
    assert r.returncode == 0, r.stderr
    assert rep["passed"] and rep["max_abs_error_vs_exact"] < 1e-6


def test_refresh_inside_a_deep_chain(tmp_path):
    ok = run_program(os.path.join(GOLDEN, "packed_refresh_v2.txt"), str(tmp_path / "r.json"), 1e-3, 1e-3,
                     log_n=12, bootstrap_passes=2)
    rep = json.loads((tmp_path / "r.json").read_text())
    assert ok and rep["passed"]
    assert rep["bootstraps"] >= 2 and rep["logical_refreshes"] >= 1


def test_gate_failure_exit_code(tmp_path):
    r, rep = _run_cli(tmp_path, "packed_linear_v2.txt", 1e-30, 1e-30)
    assert r.returncode == 1 and rep["passed"] is False


def test_bad_arguments_exit_code(tmp_path):
    r, _ = _run_cli(tmp_path, "packed_linear_v2.txt", 1e-6, 1e-6, "--no-such-flag")
    assert r.returncode == 2 and "unknown packed option" in r.stderr


def test_mamba3_siso_generation(tmp_path):
    """A 2-layer Mamba-3 SISO model (random init, d_model 64, d_state 16)
    compiled by the reference's exporter path (tests/golden/make_mamba3_program.py):
    3 prompt tokens and 2 client-feedback steps, where the client decrypts the
    final hidden vector, picks the greedy token with the tied head and feeds
    its embedding back (three generated tokens).  The tokens must equal the
    reference's polynomial and exact paths and every output must stay within
    1e-2 of both references."""
    with open(os.path.join(GOLDEN, "mamba3_tokens.json")) as f:
        want = json.load(f)
    r, rep = _run_cli(tmp_path, "packed_mamba3_siso_v2.txt", 1e-2, 1e-2, "--client-head",
                      os.path.join(GOLDEN, "mamba3_client_head.f32"))
    assert r.returncode == 0, r.stderr
    assert rep["passed"] and rep["non_finite"] == 0
    assert rep["generated_token_ids"] == want["polynomial_token_ids"] == want["exact_token_ids"]
    assert rep["bootstraps"] > 0


def test_classical128_mode(tmp_path):
    """--security 128-classic as the reference's executable sets it up: ring
    2^17, four HYBRID digits, the program's 256 slots sparsely packed (so
    bootstrapping runs the sparse-packing trace), and the Q*P audit (45 Q + 12
    P primes, 3376 bits, within the 3523-bit classical-128 bound for 2^17)
    written beside the result."""
    out = tmp_path / "native.json"
    r = subprocess.run([CLI, os.path.join(GOLDEN, "packed_refresh_v2.txt"), str(out), "1e-3", "1e-3",
                        "--security", "128-classic"], capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr
    assert "classical128 ring=131072 QP_bits=3376 bound=3523 digits=4" in r.stdout
    rep = json.loads(out.read_text())
    audit = json.loads((tmp_path / "native.json.parameters.json").read_text())
    assert rep["passed"] and rep["security"] == "128-classic" and rep["ring_dimension"] == 131072
    assert rep["slots"] == 256 and rep["bootstraps"] >= 2
    assert rep["security_audit"] == audit and audit["passed"] and audit["qp_bits"] == 3376
    assert audit["q_towers"] == 45 and audit["p_towers"] == 12 and audit["hybrid_digits"] == 4


def test_security_digits_need_classical128(tmp_path):
    r, _ = _run_cli(tmp_path, "packed_linear_v2.txt", 1e-6, 1e-6, "--security-digits", "4")
    assert r.returncode == 2
