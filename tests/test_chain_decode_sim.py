"""The encrypted chain decode's host schedule (EncryptedChain / run_chain:
masks, rotations, level budgeting, refresh points and bounds, the client loop)
on the slot-level model of the CryptoContext API (tests/slot_sim.py), against
the reference exporter's polynomial-circuit references.  Without bootstrap
noise the schedule must reproduce the references to float32 rounding; with
noise of the two-pass refresh's measured size (1e-6 x bound) its error is the
estimate the GPU test's tolerance is set from.  No GPU."""
import os

import numpy as np
import pytest

from conftest import GOLDEN
from fhe_mamba_b200.chain_payload import read_chain_payload, run_chain
from slot_sim import SimError, SlotContext

CHAIN = os.path.join(GOLDEN, "mamba2_chain")
JOINT = os.path.join(GOLDEN, "mamba2_chain_joint")


@pytest.fixture(scope="module")
def payload():
    return read_chain_payload(CHAIN)


def test_schedule_is_exact_without_noise(payload):
    cc = SlotContext(2048, refresh_noise=0.0)
    r = run_chain(cc, payload, 3, 1e-4)
    m = r["measurements"]
    assert r["passed"] and m["correctness_reference"] == "polynomial-circuit"
    assert m["max_abs_error"] < 1e-5  # float32 references
    assert m["refreshes"] == cc.refresh_count >= 6
    assert cc.max_refresh_ratio <= 1.0


def test_schedule_with_refresh_noise(payload):
    cc = SlotContext(2048, refresh_noise=1e-6)
    r = run_chain(cc, payload, 3, 1e-3)
    assert r["passed"] and r["measurements"]["max_abs_error"] < 1e-3
    assert np.isfinite(r["measurements"]["max_abs_error_vs_exact"])
    # the bounds come from calibration sequences, carried bounds and domains,
    # not from these test inputs, and still cover them
    assert cc.max_refresh_ratio <= 1.0


def test_client_loop(payload):
    cc = SlotContext(2048, refresh_noise=1e-6)
    r = run_chain(cc, payload, 3, 1e-3, autoregressive_client_loop=True)
    m = r["measurements"]
    assert r["passed"] and m["autoregressive_tokens_match"]
    assert m["autoregressive_selected_ids"] == payload.autoregressive["poly_generated_ids"] == [80, 117]


def test_cut_chain_compares_the_last_layer():
    p = read_chain_payload(CHAIN, max_layers=1, autoregressive=False)
    r = run_chain(SlotContext(2048, refresh_noise=0.0), p, 2, 1e-4)
    assert r["passed"] and r["parameters"]["layers"] == 1 and r["measurements"]["max_abs_error"] < 1e-5


@pytest.mark.parametrize("left", [22, 19, 15])
def test_fewer_levels_after_refresh(payload, left):
    """Bootstrap level budgets other than {4, 4} return fewer levels; the
    schedule refreshes more often and stays exact."""
    cc = SlotContext(2048, refresh_left=left, refresh_noise=0.0)
    assert run_chain(cc, payload, 2, 1e-4)["passed"]


def test_token_count_checks(payload):
    with pytest.raises(ValueError, match="exceeds n_test_tokens"):
        run_chain(SlotContext(2048), payload, 4)
    with pytest.raises(ValueError, match="autoregressive server evaluations"):
        run_chain(SlotContext(2048), payload, 4, autoregressive_client_loop=True)


def test_simulator_catches_missing_keys_and_bounds():
    cc = SlotContext(16)
    ct = cc.Encrypt(cc.MakeCKKSPackedPlaintext(np.arange(16.0)))
    with pytest.raises(SimError, match="missing rotation key"):
        cc.EvalRotate(ct, 3)
    with pytest.raises(SimError, match="x its bound"):
        cc.refresh(ct, 10.0)
    x = ct
    for _ in range(cc.n_q - 1):
        x = cc.EvalMult(x, 1.5)
    with pytest.raises(SimError, match="underflow"):
        cc.EvalMult(x, 1.5)


class _CountingContext(SlotContext):
    """Records the pass count of every refresh by the bound it was given."""

    def __init__(self, *a, **k):
        super().__init__(*a, **k)
        self.passes_seen = []

    def refresh(self, ct, bound=1.0, passes=2, merge=False):
        self.passes_seen.append(passes)
        return super().refresh(ct, bound, passes)


@pytest.mark.parametrize("meta_bts,residual_layers", [(False, ()), (True, ()), (True, (1,))])
def test_meta_bts_policy(payload, meta_bts, residual_layers):
    """The reference decode's selective Meta-BTS: with it off every refresh is
    one bootstrap (this payload has no scheduled normalization); with it on,
    only carried values, the gated norm's polynomial input and the selected
    layers' residual refreshes are two-pass (here: the gated values, 6 of the
    ~25 refreshes; the carried values never run out of levels)."""
    from fhe_mamba_b200.chain_payload import meta_bts_policy
    cc = _CountingContext(2048, refresh_noise=0.0)
    r = run_chain(cc, payload, 3, 1e-4, meta_bts=meta_bts, meta_bts_residual_layers=residual_layers)
    m = r["measurements"]
    assert r["passed"] and m["refreshes"] == len(cc.passes_seen)
    assert m["meta_bts_applied"] == cc.passes_seen.count(2)
    if not meta_bts:
        assert m["meta_bts_applied"] == 0
    else:
        assert 0 < m["meta_bts_applied"] < m["refreshes"]
    policy = meta_bts_policy(1, meta_bts, residual_layers)
    assert policy("state") == policy("xbc") == policy("g") == policy("n2_v") == (2 if meta_bts else 1)
    assert policy("proj") == policy("n1_y") == 1
    assert policy("h") == (2 if 1 in residual_layers else 1)
    assert meta_bts_policy(0, False, (), scheduled=True)("proj") == 2
    assert meta_bts_policy(0, False, (), scheduled=True)("state") == 1


def test_every_refresh_two_pass_by_default(payload):
    cc = _CountingContext(2048, refresh_noise=0.0)
    r = run_chain(cc, payload, 2, 1e-4)
    assert set(cc.passes_seen) == {2} and r["measurements"]["meta_bts_applied"] == r["measurements"]["refreshes"]


def test_joint_payload_schedule():
    """Joint gates (a per-head coefficient basis), degree-768/384 SiLU fits and
    scheduled inverse square roots (12-13 coupled steps, per-step refresh
    bounds) through the same layer."""
    p = read_chain_payload(JOINT)
    cc = SlotContext(2048, refresh_noise=0.0)
    r = run_chain(cc, p, 3, 1e-4)
    assert r["passed"] and r["measurements"]["max_abs_error"] < 1e-5 and cc.max_refresh_ratio <= 1.0
    cc = SlotContext(2048, refresh_noise=1e-6)
    r = run_chain(cc, p, 3, 1e-3)
    assert r["passed"], r["measurements"]["max_abs_error"]
    assert cc.max_refresh_ratio <= 1.0  # data-free bounds (no embedding table in this payload)


def test_joint_payload_reference_policy():
    """Scheduled-normalization layers make every transient refresh two-pass
    under the reference's policy, even with Meta-BTS off."""
    p = read_chain_payload(JOINT)
    cc = _CountingContext(2048, refresh_noise=0.0)
    r = run_chain(cc, p, 2, 1e-4, meta_bts=False)
    assert r["passed"] and r["measurements"]["meta_bts_applied"] == cc.passes_seen.count(2) > 0


def test_process_separated_roles(tmp_path):
    """client-init / server-eval / client-decrypt through the handoff directory
    (the reference's protocol): the server loads only evaluation keys and
    cannot decrypt; the client checks the outputs; a second client-init into a
    used directory is refused."""
    from fhe_mamba_b200 import mamba2_decode
    root = tmp_path / "handoff"
    servers = []

    def factory():
        cc = SlotContext(2048, refresh_noise=0.0)
        servers.append(cc)
        return cc

    base = ["--input-chain", CHAIN, "--output-json", str(tmp_path / "r.json"), "--ring-dim", "4096",
            "--security", "not-set", "--tokens", "3", "--tolerance", "1e-4", "--handoff-dir", str(root)]
    init = mamba2_decode.run(mamba2_decode.parse_args(base + ["--process-role", "client-init"]), factory)
    assert init["passed"] and init["measurements"]["encrypted_inputs_written"] == 3
    assert sorted(p.name for p in (root / "exchange").iterdir()) == [f"input_t{t}.ct.npz" for t in range(3)]
    assert oct((root / "client").stat().st_mode & 0o777) == "0o700"
    server = mamba2_decode.run(mamba2_decode.parse_args(base + ["--process-role", "server-eval"]), factory)
    assert server["passed"] and not servers[-1].has_secret and server["measurements"]["refreshes"] > 0
    with pytest.raises(SimError, match="no secret"):
        servers[-1].Decrypt(servers[-1].DeserializeCiphertext(root / "exchange" / "output_t0.ct"))
    client = mamba2_decode.run(mamba2_decode.parse_args(base + ["--process-role", "client-decrypt"]), factory)
    m = client["measurements"]
    assert client["passed"] and m["max_abs_error"] < 1e-5 and m["per_token_decrypt_ok"] == [1, 1, 1]
    assert m["server_secret_key_files"] == 0
    with pytest.raises(ValueError, match="non-empty handoff root"):
        mamba2_decode.run(mamba2_decode.parse_args(base + ["--process-role", "client-init"]), factory)
    # a secret that leaks into server/ fails the check
    (root / "server" / "client.keys").write_bytes(b"x")
    leaked = mamba2_decode.run(mamba2_decode.parse_args(base + ["--process-role", "client-decrypt"]), factory)
    assert not leaked["passed"] and leaked["measurements"]["server_secret_key_files"] == 1


def test_single_layer_mode_and_layer_errors(tmp_path):
    """--input LAYER_DIR (one m1 payload: its test inputs in, its test outputs
    as the reference, no final norm) and --debug-layer-errors (every layer's
    decrypted output against that layer's polynomial reference)."""
    from fhe_mamba_b200 import mamba2_decode
    from fhe_mamba_b200.chain_payload import read_layer_as_chain
    p = read_layer_as_chain(os.path.join(CHAIN, "layer_01"))
    assert not p.full_chain and not p.chain_mode and p.n_test_tokens == 3
    r = run_chain(SlotContext(2048, refresh_noise=0.0), p, 3, 1e-4)
    assert r["passed"] and r["measurements"]["correctness_reference"] == "polynomial-circuit"
    args = mamba2_decode.parse_args(["--input", os.path.join(CHAIN, "layer_00"), "--output-json",
                                     str(tmp_path / "r.json"), "--security", "not-set", "--tokens", "2"])
    assert mamba2_decode.run(args, lambda: SlotContext(2048, refresh_noise=0.0))["passed"]
    full = read_chain_payload(CHAIN)
    r = run_chain(SlotContext(2048, refresh_noise=0.0), full, 3, 1e-4, debug_layer_errors=True)
    per_layer = r["measurements"]["per_token_layer_max_abs_error"]
    assert len(per_layer) == 3 and all(len(row) == 2 and max(row) < 1e-4 for row in per_layer)
