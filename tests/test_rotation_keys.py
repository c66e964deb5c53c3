"""Rotation-key plans (fhe_mamba_b200/rotation_keys.py): NAF digits against
the reference's own (tests/golden/rotation_naf.json), the three plan modes,
and the chain decode under compact and balanced plans on the slot-level model
(every composite rotation must find its keys; results stay exact).  No GPU."""
import json
import os
from itertools import pairwise

import numpy as np
import pytest

from conftest import GOLDEN
from fhe_mamba_b200.rotation_keys import canonical_rotation, key_bytes, naf, plan_keys


def test_naf_matches_reference():
    with open(os.path.join(GOLDEN, "rotation_naf.json")) as f:
        golden = json.load(f)
    for value, steps in golden.items():
        assert naf(int(value)) == steps, value
    for value in range(-5000, 5001):
        steps = naf(value)
        assert sum(steps) == value
        ks = sorted(abs(s).bit_length() for s in steps)
        assert all(b - a >= 2 for a, b in pairwise(ks))


def test_canonical_rotation():
    assert canonical_rotation(3, 16) == 3 and canonical_rotation(9, 16) == -7 and canonical_rotation(8, 16) == 8
    assert canonical_rotation(-8, 16) == 8 and canonical_rotation(32, 16) == 0
    with pytest.raises(ValueError):
        canonical_rotation(1, 12)


def test_plan_modes():
    slots = 1 << 11
    freqs = {3: 10.0, 7: 1.0, 100: 5.0, 511: 8.0, 2: 3.0, -1792 % slots: 6.0}
    full = plan_keys(freqs, slots, "full")
    assert set(full.keys) == {3, 7, 100, 511, 2, canonical_rotation(-1792, slots)}
    assert full.stats["rotation_overhead_factor"] == 1.0
    compact = plan_keys(freqs, slots, "compact")
    assert all(abs(k) & (abs(k) - 1) == 0 for k in compact.keys)  # signed powers of two only
    for i in freqs:
        assert sum(compact.steps(i)) == canonical_rotation(i, slots)
        assert all(s in compact.direct for s in compact.steps(i))
    assert compact.stats["rotation_overhead_factor"] > 1.0
    per = key_bytes(1 << 12, 57, 4)
    assert per == 2 * 4 * 57 * 4096 * 8
    # a budget of the base plus two keys takes the two largest savings
    balanced = plan_keys(freqs, slots, "balanced", (len(compact.keys) + 2) * per, per)
    extra = set(balanced.keys) - set(compact.keys)
    assert extra == {3, 100}  # savings 10 x (2 - 1) and 5 x (3 - 1) beat 511: 8 x (2 - 1)
    assert compact.stats["rotation_overhead_factor"] > balanced.stats["rotation_overhead_factor"] > 1.0
    required = plan_keys(freqs, slots, "compact", required=[7])
    assert 7 in required.direct and required.steps(7) == [7]
    with pytest.raises(ValueError, match="balanced plan needs"):
        plan_keys(freqs, slots, "balanced")
    with pytest.raises(ValueError, match="rotation-keys"):
        plan_keys(freqs, slots, "sparse")


@pytest.mark.parametrize("mode", ["compact", "balanced"])
def test_chain_decode_under_key_plans(mode):
    from fhe_mamba_b200.chain_payload import read_chain_payload, run_chain
    from slot_sim import SlotContext
    p = read_chain_payload(os.path.join(GOLDEN, "mamba2_chain"))
    full_cc = SlotContext(2048, refresh_noise=0.0)
    full = run_chain(full_cc, p, 2, 1e-4)
    cc = SlotContext(2048, refresh_noise=0.0)
    r = run_chain(cc, p, 2, 1e-4, rotation_keys=mode, rotation_key_gib=0.05)
    m = r["measurements"]
    assert r["passed"] and m["max_abs_error"] < 1e-5
    assert m["rotation_keys"] < full["measurements"]["rotation_keys"] and len(cc.keys) == m["rotation_keys"]
    assert m["composite_rotation_applications"] > 0
    assert m["rotation_key_plan"]["mode"] == mode
