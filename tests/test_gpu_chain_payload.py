"""The reference exporter's Mamba-2 chain payload (tests/golden/mamba2_chain:
2 layers, d_model 64, 16 heads x 8, d_state 32, degree-96/64/24 activations,
degree-47/31 Newton-refined inverse square roots) decoded on ciphertexts:
the decrypted final hidden vectors against the exporter's polynomial-circuit
references (chain_expected_poly_final), and the client loop's greedy ids.
Measured on a B200: 2.5e-6, the float32 rounding of the references
themselves; the tolerance is the error the slot-level model of the same
schedule predicts with the two-pass refresh's noise bound (1e-6 x the refresh
bound, test_chain_decode_sim)."""
import json
import os

import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu

CHAIN = os.path.join(GOLDEN, "mamba2_chain")
TOL = 1e-4


def test_chain_decode_matches_polynomial_circuit():
    from fhe_mamba_b200 import CCParams, CryptoContext
    from fhe_mamba_b200.chain_payload import read_chain_payload, run_chain
    p = read_chain_payload(CHAIN)
    cc = CryptoContext(CCParams(ring_dim=1 << 12, multiplicative_depth=44, scaling_mod_size=59,
                                first_mod_size=60, num_large_digits=3))
    cc.KeyGen(53)
    cc.EvalBootstrapSetup((4, 4))
    cc.EvalBootstrapKeyGen()
    r = run_chain(cc, p, 3, TOL)
    m = r["measurements"]
    print("chain decode", m["per_token_max_abs_error"], "refreshes", m["refreshes"],
          "s/token", m["seconds_per_token"])
    assert r["passed"], m
    assert m["max_abs_error"] < TOL and m["refreshes"] >= 6


def test_cli_client_loop(tmp_path):
    from fhe_mamba_b200 import mamba2_decode
    out = tmp_path / "result.json"
    rc = mamba2_decode.main(["--input-chain", CHAIN, "--output-json", str(out), "--ring-dim", "4096",
                             "--security", "not-set", "--bootstrap-level-budget-cts", "4",
                             "--bootstrap-level-budget-stc", "4", "--autoregressive-client-loop", "1",
                             "--tokens", "3", "--tolerance", str(TOL), "--seed", "59"])
    r = json.loads(out.read_text())
    print("client loop", r.get("measurements", r))
    assert rc == 0 and r["passed"], r
    assert r["measurements"]["autoregressive_selected_ids"] == [80, 117]
    assert r["parameters"]["num_large_digits"] == 3


def test_reference_refresh_policy():
    """The reference decode's own refresh policy (--meta-bts 1: two-pass only
    for carried values and the gated norm's input, single bootstraps
    elsewhere).  Measured on a B200: 2.8e-4 (8.4e-4 with Meta-BTS off) against
    2.6e-6 when every refresh is two-pass; the bound keeps a 7x margin."""
    from fhe_mamba_b200 import CCParams, CryptoContext
    from fhe_mamba_b200.chain_payload import read_chain_payload, run_chain
    p = read_chain_payload(CHAIN)
    cc = CryptoContext(CCParams(ring_dim=1 << 12, multiplicative_depth=44, scaling_mod_size=59,
                                first_mod_size=60, num_large_digits=3))
    cc.KeyGen(67)
    cc.EvalBootstrapSetup((4, 4))
    cc.EvalBootstrapKeyGen()
    r = run_chain(cc, p, 3, 2e-3, meta_bts=True)
    m = r["measurements"]
    print("meta-bts policy", m["max_abs_error"], m["refreshes"], m["meta_bts_applied"])
    assert r["passed"], m
    assert 0 < m["meta_bts_applied"] < m["refreshes"]


def test_joint_payload_decode():
    """The joint format (tests/golden/mamba2_chain_joint): shared-dissipation
    gates on a per-head coefficient basis, degree-768/384 SiLU fits, scheduled
    inverse square roots with a dedicated final norm.  Measured on a B200:
    5.6e-6 (the references' float32 floor), 75 refreshes over 3 tokens."""
    from fhe_mamba_b200 import CCParams, CryptoContext
    from fhe_mamba_b200.chain_payload import read_chain_payload, run_chain
    p = read_chain_payload(os.path.join(GOLDEN, "mamba2_chain_joint"))
    cc = CryptoContext(CCParams(ring_dim=1 << 12, multiplicative_depth=44, scaling_mod_size=59,
                                first_mod_size=60, num_large_digits=3))
    cc.KeyGen(71)
    cc.EvalBootstrapSetup((4, 4))
    cc.EvalBootstrapKeyGen()
    r = run_chain(cc, p, 3, TOL)
    m = r["measurements"]
    print("joint decode", m["per_token_max_abs_error"], "refreshes", m["refreshes"], "s/token",
          m["seconds_per_token"])
    assert r["passed"], m


def test_process_separated_decode(tmp_path):
    """The reference's three-process protocol, each role its own process:
    client-init (keys, encrypted inputs), server-eval (evaluation keys only),
    client-decrypt (checks the outputs against the polynomial circuit)."""
    import subprocess
    import sys
    root = tmp_path / "handoff"
    base = [sys.executable, "-m", "fhe_mamba_b200.mamba2_decode", "--input-chain", CHAIN, "--ring-dim", "4096",
            "--security", "not-set", "--bootstrap-level-budget-cts", "4", "--bootstrap-level-budget-stc", "4",
            "--tokens", "2", "--tolerance", str(TOL), "--handoff-dir", str(root), "--seed", "73"]
    results = {}
    for role in ("client-init", "server-eval", "client-decrypt"):
        out = tmp_path / f"{role}.json"
        proc = subprocess.run(base + ["--process-role", role, "--output-json", str(out)], capture_output=True,
                              text=True, timeout=600)
        results[role] = json.loads(out.read_text())
        assert proc.returncode == 0, (role, results[role], proc.stderr[-2000:])
    m = results["client-decrypt"]["measurements"]
    print("process-separated decode", m["per_token_max_abs_error"],
          results["server-eval"]["measurements"]["token_step_seconds"])
    assert m["max_abs_error"] < TOL and m["per_token_decrypt_ok"] == [1, 1] and m["server_secret_key_files"] == 0
    assert results["server-eval"]["measurement_scope"]["server_secret_key_loaded"] is False


def test_compact_rotation_keys():
    """The compact key plan: only signed powers of two (plus the fused
    transforms' steps) are keyed, every other rotation is composed.  Measured
    on a B200: 2.6e-6 with 33 instead of 53 keys, 336 composed key
    applications over 2 tokens, 0.51 s per token (0.40 with every key)."""
    from fhe_mamba_b200 import CCParams, CryptoContext
    from fhe_mamba_b200.chain_payload import read_chain_payload, run_chain
    p = read_chain_payload(CHAIN)
    cc = CryptoContext(CCParams(ring_dim=1 << 12, multiplicative_depth=44, scaling_mod_size=59,
                                first_mod_size=60, num_large_digits=3))
    cc.KeyGen(79)
    cc.EvalBootstrapSetup((4, 4))
    cc.EvalBootstrapKeyGen()
    r = run_chain(cc, p, 2, TOL, rotation_keys="compact")
    m = r["measurements"]
    assert r["passed"], m
    assert m["composite_rotation_applications"] > 0 and m["rotation_key_plan"]["mode"] == "compact"
