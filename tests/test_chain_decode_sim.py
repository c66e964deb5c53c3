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
    assert r["measurements"]["max_abs_error_vs_exact"] > r["measurements"]["max_abs_error"]


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
